// MLA attention core of DeepSeek-V2-Lite prefill (the causal scaled-dot-product attention of
// src/reference/mla.py:355-378 with 192-wide q/k heads = 128 nope + 64 RoPE, 128-wide v
// heads), and the whole MLA forward around it (src/reference/mla.py:295-393):
//
//   qkv   = x @ [W_q; W_kv_a]^T            one tcgen05 GEMM: [M, heads*192 + 512 + 64]
//   lat   = RMSNorm(qkv[:, heads*192 : +512])
//   kv    = lat @ W_kv_b^T                  [M, heads*(128 + 128)]  (k_nope | v per head)
//   RoPE in place on the 64-wide q_pe of every head and on k_pe inside qkv
//   o     = causal softmax(q k^T * scale) v  (this file's attention kernel), [M, heads*128]
//   out   = o @ W_o^T                        [M, hidden]
//
// Attention kernel (one CTA per (batch, head, 128-row q tile), 192 threads):
//   warp 0       TMA producer of Q and K: the Q tile once (3 boxes of 128 rows x 64
//                columns: nope, nope, rope, straight out of qkv), then per 128-row kv block
//                the K tile (k_nope 2 boxes from kv, k_pe 1 box from qkv, shared by the
//                heads) into a 2-stage ring (128-byte swizzle).
//   warp 10      TMA producer of the V tiles (2 boxes per block: 128 kv rows x 64 dims of
//                the v half of kv, 2-stage ring), so a K load never waits behind a V stage.
//   warp 1       MMA issuer (one thread): S_j = Q K_j^T (M=128, N=128, K=192) into one of two
//                TMEM buffers, then O += P_{j-1} V_{j-1} (M=128, N=128, K=128) with P read
//                from TMEM (the softmax warps write it over S) and V read straight from
//                the kv rows as an MN-major B operand (no transposed copy).
//   warps 2-9    softmax, two warps per 32-row TMEM quarter, each thread one row's 64 of the
//                128 S values of a block (the pair exchanges row maxima through shared
//                memory): row max (log2 domain), P_j = 2^(s*scale - m) rounded to bf16 into
//                the S buffer's first 64 columns, running sum; m is raised (and the O
//                accumulator in TMEM rescaled by 2^(m_old - m_new)) only when the row max
//                grows by more than 2^8, so most blocks leave O alone; at the end O / l ->
//                bf16 -> out.
// CTAs are ordered (batch, head)-major, longest q tile first within a head.  Every wait is
// bounded; a wait that runs out sets the device status and the kernel drains and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstring>
#include <mutex>

#include "kernels.cuh"
#include "ptx.cuh"

namespace ds {
namespace attn {
namespace {

constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int kThreads = 352;  // K producer, MMA, 8 softmax warps, V producer
constexpr uint32_t CHUNK = 128 * 64 * 2;  // one 128-row x 64-column bf16 box: 16 KiB
constexpr uint32_t Q_BYTES = 3 * CHUNK;
constexpr uint32_t K_BYTES = 3 * CHUNK;
constexpr uint32_t V_BYTES = 2 * CHUNK;
constexpr int STAGES = 2;
constexpr uint32_t kTileBytes = Q_BYTES + STAGES * (K_BYTES + V_BYTES);  // 208 KiB
constexpr uint32_t kTailBytes = 256 + 6 * 128 * 4 + 128;  // barriers, then the softmax pairs' exchange
constexpr size_t kSmemBytes = 1024 + kTileBytes + kTailBytes;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSCol0 = 0, kSCol1 = 128, kOCol0 = 256, kOCol1 = 384;  // O per tile parity
constexpr long long kTimeoutCycles = 4000000000LL;

struct Params {
  int batch, seq, heads;
  int krope_col;        // column of k_pe in qkv
  float scale_log2;     // softmax scale * log2(e)
  __nv_bfloat16* out;   // [batch*seq, heads*128]
  int ldo;
  int* tile_counter;  // zero at launch: the next tile to hand out
  int* status;
};

__device__ __forceinline__ uint32_t pack_bf16(float a, float b, float& ra, float& rb) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float2 f = __bfloat1622float2(h);
  ra = f.x;
  rb = f.y;
  return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void __launch_bounds__(kThreads, 1)
    mla_attention_kernel(const __grid_constant__ CUtensorMap tmQ,   // qkv [B*S, ldq]
                         const __grid_constant__ CUtensorMap tmKV,  // kv [B*S, heads*256]
                         const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sQ = ptx::smem_u32(smem);
  const uint32_t sK = sQ + Q_BYTES;
  const uint32_t sV = sK + STAGES * K_BYTES;
  uint8_t* tail = smem + kTileBytes;
  const uint32_t bar0 = ptx::smem_u32(tail);
  // barriers (8 bytes each): q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2],
  // p_ready[2], o_done, drain, q_empty, o_free[2], tile_full[2], tile_empty[2].  Block barriers alternate by the CTA's
  // running block count g (over all its tiles): the softmax warps may finish block g+1
  // before the MMA thread has seen block g's phase, and a barrier that moved two phases past
  // its waiter would read as not yet complete.
  const uint32_t q_full = bar0;
  const uint32_t k_full0 = bar0 + 8, k_empty0 = bar0 + 24;
  const uint32_t v_full0 = bar0 + 40, v_empty0 = bar0 + 56;
  const uint32_t s_full0 = bar0 + 72;
  const uint32_t p_ready0 = bar0 + 88, o_done = bar0 + 104, drain_bar = bar0 + 112;
  const uint32_t q_empty = bar0 + 120, o_free0 = bar0 + 128;
  const uint32_t tile_full0 = bar0 + 144, tile_empty0 = bar0 + 160;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tail + 176);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tail + 180);
  volatile int* never_flag = reinterpret_cast<volatile int*>(tail + 184);
  volatile int* tile_slot = reinterpret_cast<volatile int*>(tail + 192);  // [2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ntq = (p.seq + BQ - 1) / BQ;
  const int ntiles = ntq * p.batch * p.heads;
  // tile k: (batch, head)-major so that the tiles in flight on the GPU at any time share a
  // few heads' K / V tiles through L2; within a head the longest tiles (most kv blocks)
  // first.  Tiles are handed out in that order by a global counter: the K producer of a CTA
  // takes the next one when it is ready for it and passes it to the CTA's other roles
  // through a 2-slot ring (tile_full / tile_empty; -1 = no more tiles).
  struct Tile {
    int h, qt, q0, nblk, row0;
  };
  auto tile_of = [&](int k) {
    Tile t;
    const int bh = k / ntq;
    t.qt = ntq - 1 - (k - bh * ntq);
    const int b = bh / p.heads;
    t.h = bh - b * p.heads;
    t.q0 = t.qt * BQ;
    t.nblk = t.qt + 1;  // causal: kv blocks 0..qt
    t.row0 = b * p.seq;
    return t;
  };
  // the MMA thread, the V producer and the eight softmax warps release a slot
  constexpr uint32_t kTileConsumers = 10;
  auto take_tile = [&](int i, int& k) -> bool {  // one thread of a consumer role
    const int sl = i & 1;
    if (!ptx::mbar_wait(tile_full0 + 8u * sl, (i >> 1) & 1, abort_flag, p.status,
                        kTimeoutCycles, DS_ERR_TIMEOUT))
      return false;
    k = tile_slot[sl];
    ptx::mbar_arrive(tile_empty0 + 8u * sl);
    return true;
  };

  if (threadIdx.x == 0) {
    ptx::mbar_init(q_full, 1);
    ptx::mbar_init(q_empty, 1);
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(k_full0 + 8u * s, 1);
      ptx::mbar_init(k_empty0 + 8u * s, 1);
      ptx::mbar_init(v_full0 + 8u * s, 1);
      ptx::mbar_init(v_empty0 + 8u * s, 1);
      ptx::mbar_init(s_full0 + 8u * s, 1);
      ptx::mbar_init(p_ready0 + 8u * s, 8);
      ptx::mbar_init(o_free0 + 8u * s, 8);
    }
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(tile_full0 + 8u * s, 1);
      ptx::mbar_init(tile_empty0 + 8u * s, kTileConsumers);
    }
    ptx::mbar_init(o_done, 1);
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *never_flag = 0;
    ptx::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmQ);
    ptx::prefetch_tmap(&tmKV);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0 || warp == 10) {
    // ------------------------------------------------------------------ TMA producers
    // warp 0: per tile its Q (once the previous tile's last S MMA has read the Q buffer),
    // then the K tiles (each waits only for the S MMA of the block two back); warp 10: the
    // V tiles (each waits for the P V of the block two back).  Both run ahead into the next
    // tile while the current one finishes.
    if (lane == 0) {
      const bool is_k = warp == 0;
      const uint32_t full0 = is_k ? k_full0 : v_full0;
      const uint32_t empty0 = is_k ? k_empty0 : v_empty0;
      int g = 0, ti = 0, q_issued = 0;
      bool ok = true;
      for (;; ++ti) {
        int k = -1;
        if (is_k) {  // fetch the next tile into slot ti & 1 once its previous use is released
          const int sl = ti & 1;
          if (!ptx::mbar_wait(tile_empty0 + 8u * sl, ((ti >> 1) & 1) ^ 1u, abort_flag, p.status,
                              kTimeoutCycles, DS_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          k = atomicAdd(p.tile_counter, 1);
          if (k >= ntiles) k = -1;
          tile_slot[sl] = k;
          ptx::mbar_arrive(tile_full0 + 8u * sl);
        } else if (!take_tile(ti, k)) {
          ok = false;
          break;
        }
        if (k < 0) break;
        const Tile t = tile_of(k);
        if (is_k) {
          if (!ptx::mbar_wait(q_empty, (ti & 1) ^ 1u, abort_flag, p.status, kTimeoutCycles,
                              DS_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(q_full, Q_BYTES);
          for (int c = 0; c < 3; ++c)
            ptx::tma_load_2d(sQ + c * CHUNK, &tmQ, q_full, t.h * 192 + c * 64, t.row0 + t.q0);
          ++q_issued;
        }
        for (int j = 0; j < t.nblk; ++j, ++g) {
          const int st = g & 1;
          if (!ptx::mbar_wait(empty0 + 8u * st, ((g >> 1) & 1) ^ 1u, abort_flag, p.status,
                              kTimeoutCycles, DS_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          const uint32_t fb = full0 + 8u * st;
          if (is_k) {
            ptx::mbar_arrive_expect_tx(fb, K_BYTES);
            const uint32_t kd = sK + st * K_BYTES;
            ptx::tma_load_2d(kd, &tmKV, fb, t.h * 256, t.row0 + j * BKV);
            ptx::tma_load_2d(kd + CHUNK, &tmKV, fb, t.h * 256 + 64, t.row0 + j * BKV);
            ptx::tma_load_2d(kd + 2 * CHUNK, &tmQ, fb, p.krope_col, t.row0 + j * BKV);
          } else {
            ptx::mbar_arrive_expect_tx(fb, V_BYTES);
            const uint32_t vd = sV + st * V_BYTES;
            // V_j: kv rows j*128 .. +127, head h's v dims 0-63 and 64-127
            ptx::tma_load_2d(vd, &tmKV, fb, t.h * 256 + 128, t.row0 + j * BKV);
            ptx::tma_load_2d(vd + CHUNK, &tmKV, fb, t.h * 256 + 192, t.row0 + j * BKV);
          }
        }
        if (!ok) break;
      }
      // every load issued here lands before the CTA exits: the last Q, the last phase of
      // each stage (a load whose stage wait failed was not issued)
      if (is_k && q_issued > 0)
        ptx::mbar_wait(q_full, (q_issued - 1) & 1, never_flag, p.status, kTimeoutCycles,
                       DS_ERR_TIMEOUT);
      for (int gg = g - 1; gg >= 0 && gg >= g - 2; --gg)
        ptx::mbar_wait(full0 + 8u * (gg & 1), (gg >> 1) & 1, never_flag, p.status,
                       kTimeoutCycles, DS_ERR_TIMEOUT);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // For block g: S_g = Q K_g^T into S buffer g & 1, then P_{g-1} V_{g-1} into the O buffer
    // of the tile (tile parity).  A tile's last P V is issued before the wait for the next
    // tile's Q, so the tile's epilogue does not wait for that load.
    if (lane == 0) {
      constexpr uint32_t idesc = ptx::idesc_bf16_f32(128, 128);
      // B = V [128 kv (K) x 128 dims (N)] MN-major: dims 0-63 of a kv row in one 128-byte
      // row of the first box, dims 64-127 one box (LBO) on; 16 kv rows per step
      constexpr uint32_t idesc_pv = ptx::idesc_bf16_f32_bmn(128, 128);
      bool ok = true;
      int g = 0, ti = 0;
      bool pending = false;             // block g-1's P V is still to be issued
      int prev_first = 0, prev_ti = 0;  // block g-1: first of its tile?, its tile index
      auto issue_pv = [&](int gp, bool first, int pti) -> bool {
        const int st = gp & 1;
        if (first) {  // overwrites O buffer pti & 1: the epilogue of tile pti - 2 is done
          if (!ptx::mbar_wait(o_free0 + 8u * (pti & 1), ((pti >> 1) & 1) ^ 1u, abort_flag,
                              p.status, kTimeoutCycles, DS_ERR_TIMEOUT))
            return false;
        }
        if (!ptx::mbar_wait(p_ready0 + 8u * st, (gp >> 1) & 1, abort_flag, p.status,
                            kTimeoutCycles, DS_ERR_TIMEOUT) ||
            !ptx::mbar_wait(v_full0 + 8u * st, (gp >> 1) & 1, abort_flag, p.status,
                            kTimeoutCycles, DS_ERR_TIMEOUT))
          return false;
        ptx::tc_fence_after();
        const uint32_t pa = tmem + (st ? kSCol1 : kSCol0);
        const uint32_t vb = sV + st * V_BYTES;
        const uint32_t od = tmem + ((pti & 1) ? kOCol1 : kOCol0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          ptx::umma_f16_ts(od, pa + kk * 8, ptx::sw128_mnmajor_desc(vb + kk * 16 * 128, CHUNK),
                           idesc_pv, (!first || kk > 0) ? 1u : 0u);
        ptx::umma_commit(v_empty0 + 8u * st);
        ptx::umma_commit(o_done);
        return true;
      };
      for (;; ++ti) {
        // the last P V of tile ti-1 first: its epilogue must not wait for tile ti's Q
        if (pending) {
          if (!issue_pv(g - 1, prev_first != 0, prev_ti)) {
            ok = false;
            break;
          }
          pending = false;
        }
        int k = -1;
        if (!take_tile(ti, k)) {
          ok = false;
          break;
        }
        if (k < 0) break;
        const Tile t = tile_of(k);
        if (!ptx::mbar_wait(q_full, ti & 1, abort_flag, p.status, kTimeoutCycles,
                            DS_ERR_TIMEOUT)) {
          ok = false;
          break;
        }
        for (int j = 0; j < t.nblk; ++j, ++g) {
          const int st = g & 1;
          if (!ptx::mbar_wait(k_full0 + 8u * st, (g >> 1) & 1, abort_flag, p.status,
                              kTimeoutCycles, DS_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t d = tmem + (st ? kSCol1 : kSCol0);
          const uint32_t kb = sK + st * K_BYTES;
#pragma unroll
          for (int kk = 0; kk < 12; ++kk) {
            const uint32_t off = (kk >> 2) * CHUNK + (kk & 3) * 32;
            ptx::umma_f16(d, ptx::sw128_kmajor_desc(sQ + off), ptx::sw128_kmajor_desc(kb + off),
                          idesc, kk > 0 ? 1u : 0u);
          }
          ptx::umma_commit(k_empty0 + 8u * st);
          ptx::umma_commit(s_full0 + 8u * st);
          if (j == t.nblk - 1) ptx::umma_commit(q_empty);  // the tile's last read of Q
          if (pending && !issue_pv(g - 1, prev_first != 0, prev_ti)) {
            ok = false;
            break;
          }
          pending = true;
          prev_first = j == 0;
          prev_ti = ti;
        }
        if (!ok) break;
      }
      if (ok && pending) issue_pv(g - 1, prev_first != 0, prev_ti);
      // no MMA may still be running when TMEM is released
      ptx::umma_commit(drain_bar);
      ptx::mbar_wait(drain_bar, 0, never_flag, p.status, kTimeoutCycles, DS_ERR_TIMEOUT);
    }
  } else {
    // ------------------------------------------------------------------ softmax (warps 2-9)
    // Two warps per 32-row TMEM quarter: `half` 0 takes S columns 0..63 (and O columns
    // 0..63), half 1 columns 64..127.  Each thread holds one row's 64 values; the pair
    // exchanges its partial row max and its wait result through shared memory (one named
    // barrier, 1 + quarter, 64 threads, per block), which also orders both warps' S loads
    // before either writes P over S.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;  // q row within the tile (= TMEM lane)
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    float* red = reinterpret_cast<float*>(tail + 256);  // [2 parity][2 half][128 rows]
    int* red_ok = reinterpret_cast<int*>(tail + 256 + 6 * 128 * 4);  // [2 parity][2 half][4]
    const uint32_t pair_bar = 1 + quarter;
    // m: the max the row's P values are taken against (log2 domain).  It is raised only when
    // the row max grows by more than kLazy (so P <= 2^kLazy), which leaves O untouched on
    // most blocks; l and O always refer to the same m, and the final O / l is exact.
    constexpr float kLazy = 8.f;
    bool ok = true;
    int g = 0, ti = 0;
    int* tile_x = reinterpret_cast<int*>(tail + 256 + 6 * 128 * 4 + 64);  // [2][2 half][4]
    // the tile loop is left only where the pair has agreed (the tile exchange below, or
    // after the sum exchange), so neither warp of a pair is left waiting in a named barrier
    for (;; ++ti) {
      int k = -1;
      if (lane == 0 && ok && !take_tile(ti, k)) k = -1;
      k = __shfl_sync(0xffffffffu, k, 0);
      tile_x[((ti & 1) * 2 + half) * 4 + quarter] = k;
      ptx::named_bar_sync(pair_bar, 64);
      k = min(k, tile_x[((ti & 1) * 2 + (half ^ 1)) * 4 + quarter]);
      if (k < 0) break;  // no more tiles, or a failed wait in either warp
      const Tile t = tile_of(k);
      const uint32_t ob = tmem + lane_off + ((ti & 1) ? kOCol1 : kOCol0) + half * 64;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < t.nblk; ++j, ++g) {
        const int st = g & 1;
        int w_ok = 0;
        if (lane == 0 && ok)
          w_ok = ptx::mbar_wait(s_full0 + 8u * st, (g >> 1) & 1, abort_flag, p.status,
                                kTimeoutCycles, DS_ERR_TIMEOUT)
                     ? 1
                     : 0;
        w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
        ptx::tc_fence_after();
        // S is read even after a failed wait (then discarded), so the pair stays in step
        const uint32_t sb = tmem + lane_off + (st ? kSCol1 : kSCol0);
        uint32_t v[2][32];
        ptx::tmem_ld32(sb + half * 64, v[0]);
        ptx::tmem_ld32(sb + half * 64 + 32, v[1]);
        ptx::tmem_wait_ld2(v[0], v[1]);
        if (j == t.qt) {  // diagonal block: kv column > q row is masked
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (half * 64 + c * 32 + i > r) v[c][i] = __float_as_uint(-INFINITY);
        }
        float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          mx0 = fmaxf(mx0, __uint_as_float(v[0][i]));
          mx1 = fmaxf(mx1, __uint_as_float(v[0][16 + i]));
          mx2 = fmaxf(mx2, __uint_as_float(v[1][i]));
          mx3 = fmaxf(mx3, __uint_as_float(v[1][16 + i]));
        }
        // exchange the partial max and the wait result (double-buffered by block parity);
        // the barrier also puts both warps' S loads before any P store below
        red[(st * 2 + half) * 128 + r] = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
        if (lane == 0) red_ok[(st * 2 + half) * 4 + quarter] = w_ok;
        ptx::tc_fence_before();
        ptx::named_bar_sync(pair_bar, 64);
        ptx::tc_fence_after();
        if (!(w_ok && red_ok[(st * 2 + (half ^ 1)) * 4 + quarter])) {  // the pair agrees
          ok = false;
          break;
        }
        const float mcand = fmaxf(red[(st * 2) * 128 + r], red[(st * 2 + 1) * 128 + r]) * p.scale_log2;
        float alpha = 1.f;
        if (mcand > m + kLazy) {
          alpha = ptx::ex2(m - mcand);  // 0 on the first block (m = -inf)
          m = mcand;
        }
        const float neg = -m;
        // P = 2^(s*scale - m) as bf16: this half's 64 values -> P columns half*32 .. +32
        float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float p0 = ptx::ex2(fmaf(__uint_as_float(v[c][2 * i]), p.scale_log2, neg));
            const float p1 = ptx::ex2(fmaf(__uint_as_float(v[c][2 * i + 1]), p.scale_log2, neg));
            sum0 += p0;
            sum1 += p1;
            const __nv_bfloat162 hp = __floats2bfloat162_rn(p0, p1);
            w[i] = *reinterpret_cast<const uint32_t*>(&hp);
          }
          ptx::tmem_st16(sb + half * 32 + c * 16, w);
        }
        l = l * alpha + (sum0 + sum1);  // this half's share of the row sum
        // The P V of block g-1 (same tile) must have landed before O is touched.  o_done is
        // waited at every block but a tile's first, in order: the P V of block g cannot start
        // before this warp's p_ready arrival and that of block g-2 finished before S_g, so
        // o_done is never more than one phase past the phase waited for.
        if (j > 0) {
          int o_ok = 1;
          if (lane == 0)
            o_ok = ptx::mbar_wait(o_done, (g - 1) & 1, abort_flag, p.status, kTimeoutCycles,
                                  DS_ERR_TIMEOUT)
                       ? 1
                       : 0;
          // a failed wait does not leave the loop here: it is carried into the next
          // block's exchange (or the tile's sum exchange), where the pair leaves together
          if (!__shfl_sync(0xffffffffu, o_ok, 0)) ok = false;
          ptx::tc_fence_after();
          if (ok && __any_sync(0xffffffffu, alpha != 1.f)) {
            uint32_t o[2][32];
            ptx::tmem_ld32(ob, o[0]);
            ptx::tmem_ld32(ob + 32, o[1]);
            ptx::tmem_wait_ld2(o[0], o[1]);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
#pragma unroll
              for (int i = 0; i < 32; ++i) o[c][i] = __float_as_uint(__uint_as_float(o[c][i]) * alpha);
              ptx::tmem_st32(ob + c * 32, o[c]);
            }
          }
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(p_ready0 + 8u * st);
      }
      // the row sum is the two halves' shares (same m); exchanged once more (a negative
      // share marks a failed warp, and the pair then leaves together)
      red[(2 * 2 + half) * 128 + r] = ok ? l : -1.f;
      ptx::named_bar_sync(pair_bar, 64);
      const float l_other = red[(2 * 2 + (half ^ 1)) * 128 + r];
      // the partner's share has been read before either warp can write the next tile's
      ptx::named_bar_sync(pair_bar, 64);
      ok = ok && __all_sync(0xffffffffu, l_other >= 0.f);
      if (!ok) break;
      int o_ok = 1;
      if (lane == 0)
        o_ok = ptx::mbar_wait(o_done, (g - 1) & 1, abort_flag, p.status, kTimeoutCycles,
                              DS_ERR_TIMEOUT)
                   ? 1
                   : 0;
      if (!__shfl_sync(0xffffffffu, o_ok, 0)) {
        ok = false;  // the next tile's first exchange takes the pair out together
        continue;
      }
      ptx::tc_fence_after();
      const float inv = 1.f / (l + l_other);
      const bool valid = t.q0 + r < p.seq;
      __nv_bfloat16* dst = p.out + static_cast<int64_t>(t.row0 + t.q0 + r) * p.ldo +
                           static_cast<int64_t>(t.h) * 128 + half * 64;
      uint32_t o[2][32];
      ptx::tmem_ld32(ob, o[0]);
      ptx::tmem_ld32(ob + 32, o[1]);
      ptx::tmem_wait_ld2(o[0], o[1]);
      // this O buffer may be overwritten by the tile after next
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(o_free0 + 8u * (ti & 1));
      if (valid) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t w[16];
          float r0, r1;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = pack_bf16(__uint_as_float(o[c][2 * i]) * inv,
                             __uint_as_float(o[c][2 * i + 1]) * inv, r0, r1);
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            d4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    }
  }

  __syncwarp();
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// RoPE in place on qkv [rows, ld]: the 64-wide q_pe of each head (columns h*192 + 128 ..) and
// k_pe (columns kcol ..): the interleave -> half transform and the rotation of
// src/reference/mla.py:176-206, out[k] = x[2k] cos[k] - x[2k+1] sin[k],
// out[32+k] = x[2k+1] cos[32+k] + x[2k] sin[32+k], one bf16 rounding.  cos/sin: bf16
// [positions, 64] tables at position pos[row] (or row % seq when pos is null).
// Four lanes per 64-wide row (lane l reads elements 16l..16l+15, i.e. pairs 8l..8l+7, and
// writes out[8l..] and out[32+8l..]); a warp covers 8 rows, each read as one 128-byte line,
// and every lane's loads complete (syncwarp) before any lane of the warp stores, so the
// in-place update never races.
__global__ void __launch_bounds__(256)
    mla_rope_inplace_kernel(__nv_bfloat16* __restrict__ qkv, int ld, int64_t rows, int seq,
                            int heads, int kcol, const __nv_bfloat16* __restrict__ cos_t,
                            const __nv_bfloat16* __restrict__ sin_t,
                            const int32_t* __restrict__ pos) {
  const int per_row = heads + 1;
  const int64_t items = rows * per_row;
  const int lane = threadIdx.x & 31;
  const int l = lane & 3;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t base = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) / 32 * 8;
       base < items; base += warps * 8) {
    const int64_t it = base + (lane >> 2);
    const bool live = it < items;
    uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0, cl = x0, ch = x0, sl = x0, sh = x0;
    __nv_bfloat16* row = nullptr;
    if (live) {
      const int64_t tok = it / per_row;
      const int hh = static_cast<int>(it - tok * per_row);
      row = qkv + tok * ld + (hh < heads ? hh * 192 + 128 : kcol);
      const uint4* x4 = reinterpret_cast<const uint4*>(row) + 2 * l;
      x0 = x4[0];
      x1 = x4[1];
      const int64_t pr = pos != nullptr ? __ldg(pos + tok) : tok % seq;
      const uint4* c4 = reinterpret_cast<const uint4*>(cos_t + pr * 64);
      const uint4* s4 = reinterpret_cast<const uint4*>(sin_t + pr * 64);
      cl = __ldg(c4 + l);
      ch = __ldg(c4 + 4 + l);
      sl = __ldg(s4 + l);
      sh = __ldg(s4 + 4 + l);
    }
    __syncwarp();
    if (live) {
      const __nv_bfloat16* xa = reinterpret_cast<const __nv_bfloat16*>(&x0);
      const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&x1);
      const __nv_bfloat16* clp = reinterpret_cast<const __nv_bfloat16*>(&cl);
      const __nv_bfloat16* chp = reinterpret_cast<const __nv_bfloat16*>(&ch);
      const __nv_bfloat16* slp = reinterpret_cast<const __nv_bfloat16*>(&sl);
      const __nv_bfloat16* shp = reinterpret_cast<const __nv_bfloat16*>(&sh);
      uint4 lo, hi;
      __nv_bfloat16* lop = reinterpret_cast<__nv_bfloat16*>(&lo);
      __nv_bfloat16* hip = reinterpret_cast<__nv_bfloat16*>(&hi);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const __nv_bfloat16* xx = q < 4 ? xa : xb;
        const float a = __bfloat162float(xx[2 * (q & 3)]);
        const float bb = __bfloat162float(xx[2 * (q & 3) + 1]);
        lop[q] = __float2bfloat16_rn(a * __bfloat162float(clp[q]) - bb * __bfloat162float(slp[q]));
        hip[q] = __float2bfloat16_rn(bb * __bfloat162float(chp[q]) + a * __bfloat162float(shp[q]));
      }
      uint4* o4 = reinterpret_cast<uint4*>(row);
      o4[l] = lo;
      o4[4 + l] = hi;
    }
  }
}

// ---- host ------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
bool g_attr_set[64] = {};
std::mutex g_attr_mutex;

int tmap_2d(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld) {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  if (g_encode == nullptr) return fail(DS_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64u, 128u};
  cuuint32_t estr[2] = {1u, 1u};
  const CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%lld cols=%lld", (int)r,
                (long long)rows, (long long)cols);
  return DS_OK;
}

}  // namespace

// Attention over qkv (RoPE already applied in place) and kv
// [batch*heads*128, seq]; out [batch*seq, heads*128].
int launch_attention(const void* qkv, int ldq, const void* kv, void* out, int batch,
                     int seq, int heads, float softmax_scale, int* tile_counter,
                     cudaStream_t s) {
  DS_REQUIRE(batch >= 1 && seq >= 1 && heads >= 1, "mla_attention: bad shape");
  DS_REQUIRE(seq % 8 == 0, "mla_attention: seq_len must be a multiple of 8");
  DS_REQUIRE(ldq % 8 == 0 && ldq >= heads * 192 + 512 + 64, "mla_attention: bad qkv stride");
  DS_REQUIRE(aligned16(qkv) && aligned16(kv) && aligned16(out),
             "mla_attention: buffers must be 16-byte aligned");
  DeviceInfo di;
  DS_TRY(device_info(&di));
  {
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    if (!g_attr_set[di.device]) {
      DS_CUDA(cudaFuncSetAttribute(mla_attention_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(kSmemBytes)));
      g_attr_set[di.device] = true;
    }
  }
  const int64_t M = static_cast<int64_t>(batch) * seq;
  CUtensorMap tq, tkv;
  DS_TRY(tmap_2d(&tq, qkv, M, ldq, ldq));
  DS_TRY(tmap_2d(&tkv, kv, M, static_cast<int64_t>(heads) * 256, static_cast<int64_t>(heads) * 256));
  Params p{};
  p.batch = batch;
  p.seq = seq;
  p.heads = heads;
  p.krope_col = heads * 192 + 512;
  p.scale_log2 = static_cast<float>(static_cast<double>(softmax_scale) * 1.4426950408889634);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = heads * 128;
  p.tile_counter = tile_counter;
  p.status = device_status_ptr();
  if (p.status == nullptr) return fail(DS_ERR_CUDA, "device status word unavailable");
  DS_REQUIRE(tile_counter != nullptr, "mla_attention: no tile counter");
  DS_CUDA(cudaMemsetAsync(tile_counter, 0, sizeof(int), s));
  // persistent: one CTA per SM (the shared memory allows no more) walks its tiles
  const int64_t ntiles = static_cast<int64_t>((seq + BQ - 1) / BQ) * batch * heads;
  DS_REQUIRE(ntiles < (int64_t(1) << 31), "mla_attention: too many tiles");
  const int grid = static_cast<int>(ntiles < di.num_sms ? ntiles : di.num_sms);
  mla_attention_kernel<<<grid, kThreads, kSmemBytes, s>>>(tq, tkv, p);
  DS_LAUNCH_CHECK("mla_attention_kernel");
  return DS_OK;
}

int launch_mla_rope(void* qkv, int ldq, int64_t rows, int seq, int heads, const void* cos_t,
                    const void* sin_t, const int32_t* pos, cudaStream_t s) {
  DeviceInfo di;
  DS_TRY(device_info(&di));
  const int64_t items = rows * (heads + 1);
  int64_t grid = (items * 4 + 255) / 256;  // four lanes per row
  if (grid > di.num_sms * 16) grid = di.num_sms * 16;
  mla_rope_inplace_kernel<<<static_cast<int>(grid > 0 ? grid : 1), 256, 0, s>>>(
      static_cast<__nv_bfloat16*>(qkv), ldq, rows, seq, heads, heads * 192 + 512,
      static_cast<const __nv_bfloat16*>(cos_t), static_cast<const __nv_bfloat16*>(sin_t), pos);
  DS_LAUNCH_CHECK("mla_rope_inplace_kernel");
  return DS_OK;
}

}  // namespace attn
}  // namespace ds

// ---- C ABI ------------------------------------------------------------------------------------
namespace {

struct MlaBuffers {
  void* qkv;  // bf16 [M, ldq]
  void* lat;  // bf16 [M, 512]
  void* kv;   // bf16 [M, heads*256]
  void* o;    // bf16 [M, heads*128]
  int* tiles;  // the attention's tile counter
};

constexpr int kLatent = 512;

int mla_ldq(int heads) { return heads * 192 + kLatent + 64; }

size_t carve_mla(ds::Carve& c, MlaBuffers* b, int batch, int seq, int heads) {
  const size_t M = static_cast<size_t>(batch) * seq;
  MlaBuffers x{};
  x.qkv = c.take<__nv_bfloat16>(M * mla_ldq(heads));
  x.lat = c.take<__nv_bfloat16>(M * kLatent);
  x.kv = c.take<__nv_bfloat16>(M * heads * 256);
  x.o = c.take<__nv_bfloat16>(M * heads * 128);
  x.tiles = c.take<int>(64);
  if (b) *b = x;
  return ds::align_up(c.used, 256);
}

ds::gemm::Problem dense_problem(const void* A, int64_t rows, int K, const void* B, int N,
                                void* out) {
  ds::gemm::Problem p{};
  p.A = A;
  p.a_rows = rows;
  p.K = K;
  p.B = B;
  p.b_rows = N;
  p.offsets = nullptr;
  p.groups = 1;
  p.n_tiles = (N + 255) / 256;
  p.seg_cols = N;
  p.b_rows_per_group = N;
  p.b_tile_stride = 256;
  p.b_half1_off = 128;
  p.weight_group_mod = 1;
  p.out = out;
  p.ldo = N;
  p.epilogue = ds::gemm::kPlain;
  return p;
}

}  // namespace

extern "C" {

size_t ds_mla_attention_workspace_size(int batch, int seq, int heads) {
  (void)batch;
  (void)seq;
  (void)heads;
  return 256;  // the tile counter (v is read in place)
}

int ds_mla_attention(const void* qkv_bf16, int qkv_ld, const void* kv_bf16, void* out_bf16,
                     int batch, int seq, int heads, float softmax_scale, void* workspace,
                     size_t workspace_bytes, void* stream) {
  DS_REQUIRE(batch >= 0 && seq >= 0 && heads >= 1, "mla_attention: bad shape");
  if (batch == 0 || seq == 0) return DS_OK;
  DS_REQUIRE(qkv_bf16 && kv_bf16 && out_bf16, "mla_attention: null pointer");
  DS_REQUIRE(workspace != nullptr && workspace_bytes >= 256 &&
                 (reinterpret_cast<uintptr_t>(workspace) & 3u) == 0,
             "mla_attention: workspace needs 256 bytes");
  return ds::attn::launch_attention(qkv_bf16, qkv_ld, kv_bf16, out_bf16, batch, seq, heads,
                                    softmax_scale, static_cast<int*>(workspace),
                                    static_cast<cudaStream_t>(stream));
}

size_t ds_mla_forward_workspace_size(int batch, int seq, int hidden, int heads) {
  (void)hidden;
  ds::Carve c(nullptr, 0);
  return carve_mla(c, nullptr, batch, seq, heads);
}

}  // extern "C"

namespace ds {
namespace dec {
int launch_cache_append(const void* src_lat, int lat_ld, const void* src_kpe, int kpe_ld,
                        int src_bstride, int batch, int n_new, int pos0, const int* pos0_dev,
                        int max_seq, int copy_raw, void* c_lat, void* c_kpe, float* c_rstd,
                        void* c_kpe_rot, const void* cos_t, const void* sin_t, float eps,
                        cudaStream_t s);
}  // namespace dec
}  // namespace ds

namespace {

struct CacheArgs {
  void* latent;
  void* kpe;
  float* rstd;
  void* kpe_rot;
  int max_seq;
  int pos0;
};

int mla_forward_impl(const void* x_bf16, const void* w_qkv_a_bf16, const float* kv_norm_weight,
                     const void* w_kv_b_bf16, const void* w_o_bf16, const void* cos_bf16,
                     const void* sin_bf16, const int32_t* positions, void* out_bf16, int batch,
                     int seq, int hidden, int heads, float eps, float softmax_scale,
                     void* workspace, size_t workspace_bytes, void** events, void* stream,
                     const CacheArgs* cache) {
  DS_REQUIRE(batch >= 0 && seq >= 0 && heads >= 1 && hidden > 0, "mla_forward: bad shape");
  DS_REQUIRE(hidden % 8 == 0, "mla_forward: hidden_size must be a multiple of 8");
  DS_REQUIRE(seq % 8 == 0 || batch * seq == 0, "mla_forward: seq_len must be a multiple of 8");
  if (batch == 0 || seq == 0) return DS_OK;
  DS_REQUIRE(x_bf16 && w_qkv_a_bf16 && kv_norm_weight && w_kv_b_bf16 && w_o_bf16 && cos_bf16 &&
                 sin_bf16 && out_bf16,
             "mla_forward: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto mark = [&](int i) -> int {
    if (events != nullptr && events[i] != nullptr)
      DS_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[i]), s));
    return DS_OK;
  };
  ds::Carve c(workspace, workspace_bytes);
  MlaBuffers b;
  carve_mla(c, &b, batch, seq, heads);
  if (!c.ok()) return ds::fail(DS_ERR_WORKSPACE, "mla_forward: workspace needs %zu bytes", c.used);
  const int64_t M = static_cast<int64_t>(batch) * seq;
  const int ldq = mla_ldq(heads);
  DS_TRY(mark(0));
  // q_proj | kv_a_proj_with_mqa in one GEMM: [M, heads*192 + 512 + 64]
  DS_TRY(ds::gemm::launch(dense_problem(x_bf16, M, hidden, w_qkv_a_bf16, ldq, b.qkv), s));
  DS_TRY(mark(1));
  DS_TRY(ds_rms_norm_strided(static_cast<const __nv_bfloat16*>(b.qkv) + heads * 192, ldq,
                             kv_norm_weight, b.lat, kLatent, static_cast<int>(M), kLatent, eps,
                             stream));
  if (cache != nullptr) {
    // the prompt's raw latents and k_pe (before the in-place RoPE below) into the cache
    const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(b.qkv);
    DS_TRY(ds::dec::launch_cache_append(q + heads * 192, ldq, q + heads * 192 + kLatent, ldq, seq,
                                        batch, seq, cache->pos0, nullptr, cache->max_seq, 1,
                                        cache->latent,
                                        cache->kpe, cache->rstd, cache->kpe_rot, cos_bf16,
                                        sin_bf16, eps, s));
  }
  DS_TRY(mark(2));
  DS_TRY(ds::gemm::launch(dense_problem(b.lat, M, kLatent, w_kv_b_bf16, heads * 256, b.kv), s));
  DS_TRY(mark(3));
  DS_TRY(ds::attn::launch_mla_rope(b.qkv, ldq, M, seq, heads, cos_bf16, sin_bf16, positions, s));
  DS_TRY(mark(4));
  DS_TRY(ds::attn::launch_attention(b.qkv, ldq, b.kv, b.o, batch, seq, heads,
                                    softmax_scale, b.tiles, s));
  DS_TRY(mark(5));
  DS_TRY(ds::gemm::launch(dense_problem(b.o, M, heads * 128, w_o_bf16, hidden, out_bf16), s));
  DS_TRY(mark(6));
  return DS_OK;
}

}  // namespace

extern "C" {

int ds_mla_forward(const void* x_bf16, const void* w_qkv_a_bf16, const float* kv_norm_weight,
                   const void* w_kv_b_bf16, const void* w_o_bf16, const void* cos_bf16,
                   const void* sin_bf16, const int32_t* positions, void* out_bf16, int batch,
                   int seq, int hidden, int heads, float eps, float softmax_scale,
                   void* workspace, size_t workspace_bytes, void** events, void* stream) {
  return mla_forward_impl(x_bf16, w_qkv_a_bf16, kv_norm_weight, w_kv_b_bf16, w_o_bf16, cos_bf16,
                          sin_bf16, positions, out_bf16, batch, seq, hidden, heads, eps,
                          softmax_scale, workspace, workspace_bytes, events, stream, nullptr);
}

int ds_mla_prefill(const void* x_bf16, const void* w_qkv_a_bf16, const float* kv_norm_weight,
                   const void* w_kv_b_bf16, const void* w_o_bf16, const void* cos_bf16,
                   const void* sin_bf16, void* out_bf16, int batch, int seq, int hidden,
                   int heads, float eps, float softmax_scale, void* cache_latent_bf16,
                   void* cache_kpe_bf16, float* cache_rstd, void* cache_kpe_rot_bf16,
                   int max_seq, int pos0, void* workspace, size_t workspace_bytes, void* stream) {
  DS_REQUIRE(pos0 == 0, "mla_prefill: the prompt starts at position 0 (pos0=%d)", pos0);
  DS_REQUIRE(seq <= max_seq, "mla_prefill: prompt longer than the cache");
  DS_REQUIRE(cache_latent_bf16 && cache_kpe_bf16 && cache_rstd && cache_kpe_rot_bf16,
             "mla_prefill: null cache pointer");
  CacheArgs c{cache_latent_bf16, cache_kpe_bf16, cache_rstd, cache_kpe_rot_bf16, max_seq, pos0};
  return mla_forward_impl(x_bf16, w_qkv_a_bf16, kv_norm_weight, w_kv_b_bf16, w_o_bf16, cos_bf16,
                          sin_bf16, nullptr, out_bf16, batch, seq, hidden, heads, eps,
                          softmax_scale, workspace, workspace_bytes, nullptr, stream, &c);
}

}  // extern "C"

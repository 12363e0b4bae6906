// MLA decode over a latent KV cache (the cache of
// src/kernels/mla_cache.py:29-219, the attention of src/reference/mla.py:295-393 for one new
// token per sequence).
//
// The cache holds, per sequence and position, the raw 512-wide latent and the raw 64-wide
// k_pe exactly as the reference's LatentKVCache stores them, plus two side arrays written
// when a token is appended: rstd = rsqrt(mean(latent^2) + eps) (the latent RMSNorm's row
// scale) and the RoPE-rotated k_pe at the token's position.  With the kv_b projection
// absorbed into the query and output weights (folded once, on the host side), a decode step
// is
//   proj  = x @ W_dec^T        W_dec = [W_qabs (heads x 512) ; W_qpe (heads x 64) ; W_kva]
//           q'_h = g * (W_uk_h^T q_nope_h) comes out directly (g: the latent norm weight)
//   append latent, k_pe, rstd, rope(k_pe) of the new token; Q = [q'_h | rope(q_pe_h)]
//   s_h(t) = rstd(t) * (q'_h . c(t)) + q_pe_h . k_pe_rot(t)            (scaled, softmax over t)
//   o_lat_h = sum_t p_h(t) rstd(t) c(t)                                 (512-wide)
//   out   = o_lat @ W_ouv^T    W_ouv_h = W_o_h W_uv_h diag(g)
// and the attention reads the cache once: it is HBM-bound (576 bf16 + 68 bytes per token).
//
// Attention kernel: one CTA per (sequence, split of the positions) and per SM, 192 threads,
// 128-token chunks streamed box by box (~167 KB of shared memory).  A chunk is nine TMA
// boxes of 128 token rows x 64 columns (latent 0..7, k_pe_rot), each with its own full and
// empty barrier: the S^T MMAs of a box are issued as soon as it lands, and a box of the next
// chunk is loaded as soon as the MMAs of this chunk that read it are done (k_pe_rot after
// S^T, latent boxes 2i and 2i+1 after the O^T block i), so the loads run under the MMAs and
// the softmax.  The MMAs have N = 16 (the heads): each costs the tensor pipe's ~46-cycle
// floor whatever M, so M = 128 tokens per S^T instruction halves their count per token.
//   warp 0   TMA producer: the sequence's Q (16 heads x 576: nine 16x64 boxes) once, then
//            per chunk the k_pe_rot box and the eight latent boxes, each once its previous
//            chunk's readers are done.
//   warp 1   MMA issuer: S^T = C Q'^T (M = 128 tokens, N = 16 heads, K = 512) and the RoPE
//            part (K = 64) into two TMEM accumulators (token r in lane r); after the softmax,
//            O^T += C^T P^T (M = 128 latent dims x 4 blocks, N = 16 heads, K = 128 tokens)
//            with the SAME latent boxes read as an MN-major A operand (no second copy of
//            the cache).
//   warps 2-5  softmax, one token per thread: s = rstd*S1 + S2 for the 16 heads, per-head
//            max over the chunk (shuffles + shared memory), lazy running max
//            (O^T rescaled in TMEM only when a head's max grows by more than 2^8), P^T (times
//            rstd) as bf16 into a 16 x 128 shared-memory tile; at the end the O^T rows (one
//            latent dim per thread), maxima and sums go to a per-split partial.
// A combine kernel merges the splits per (sequence, head) into o_lat (bf16).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <mutex>

#include "kernels.cuh"
#include "ptx.cuh"

namespace ds {
namespace dec {
namespace {

constexpr int kLatent = 512;
constexpr int kRope = 64;
constexpr int kQCols = kLatent + kRope;  // 576
constexpr int kHeads = 16;               // N of the attention MMAs
constexpr int kChunk = 128;
constexpr int kThreads = 192;
constexpr int kBoxes = 9;                      // latent 0..7, k_pe_rot
constexpr uint32_t kBox = kChunk * 64 * 2;     // 128 rows x 64 columns bf16: 16 KiB
constexpr uint32_t kQBox = 16 * 64 * 2;        // 16 rows x 64 columns: 2 KiB
constexpr uint32_t kQBytes = 9 * kQBox;        // 18 KiB
constexpr uint32_t kCBytes = kBoxes * kBox;    // 144 KiB
constexpr uint32_t kPBytes = 2 * kQBox;        // P^T: 16 heads x 128 tokens, two 16x64 atoms
constexpr uint32_t kTail = 1024;  // barriers, TMEM address, flags, then the maxima exchange
constexpr size_t kSmemBytes = 1024 + kCBytes + kQBytes + kPBytes + kTail;
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kColS1 = 0, kColS2 = 16, kColO = 32;  // O^T: 4 blocks x 16 columns
constexpr long long kTimeoutCycles = 4000000000LL;

struct Params {
  int batch, max_seq, len, nsplit, chunks_per_split;
  const int* len_dev;  // when set: the cached length before this token, read on the device
  const float* rstd;   // [batch * max_seq]
  float scale_log2;
  float* part_o;       // [batch][nsplit][16][512]
  float* part_ml;      // [batch][nsplit][2][16]: max (log2 domain), sum
  int* status;
};

__global__ void __launch_bounds__(kThreads, 1)
    mla_decode_attn_kernel(const __grid_constant__ CUtensorMap tmQ,   // Q [batch*16, 576]
                           const __grid_constant__ CUtensorMap tmC,   // latent [batch*max_seq, 512]
                           const __grid_constant__ CUtensorMap tmKr,  // k_pe_rot [batch*max_seq, 64]
                           const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sC = ptx::smem_u32(smem);        // 9 boxes: latent 0..7, k_pe_rot
  const uint32_t sQ = sC + kCBytes;               // 9 boxes of 16 x 64
  const uint32_t sP = sQ + kQBytes;               // P^T: 2 atoms of 16 x 64
  uint8_t* tail = smem + kCBytes + kQBytes + kPBytes;
  const uint32_t bar0 = ptx::smem_u32(tail);
  // barriers: box_full[9], box_empty[9], q_full, s_full, p_ready, o_done, drain
  const uint32_t box_full0 = bar0, box_empty0 = bar0 + 8 * kBoxes;
  const uint32_t q_full = bar0 + 16 * kBoxes, s_full = q_full + 8, p_ready = q_full + 16;
  const uint32_t o_done = q_full + 24, drain_bar = q_full + 32;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tail + 192);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tail + 196);
  volatile int* never_flag = reinterpret_cast<volatile int*>(tail + 200);
  float* red = reinterpret_cast<float*>(tail + 256);  // [4 warps][16 heads] per-chunk maxima
  uint8_t* sPgen = smem + kCBytes + kQBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.x / p.nsplit;
  const int split = blockIdx.x - b * p.nsplit;
  const int len = p.len_dev != nullptr ? *p.len_dev + 1 : p.len;
  const int t_begin = split * p.chunks_per_split * kChunk;
  const int t_end = min(len, t_begin + p.chunks_per_split * kChunk);
  const int nchunk = t_end > t_begin ? (t_end - t_begin + kChunk - 1) / kChunk : 0;
  const int row0 = b * p.max_seq;

  if (threadIdx.x == 0) {
    for (int c = 0; c < kBoxes; ++c) {
      ptx::mbar_init(box_full0 + 8u * c, 1);
      ptx::mbar_init(box_empty0 + 8u * c, 1);
    }
    ptx::mbar_init(q_full, 1);
    ptx::mbar_init(s_full, 1);
    ptx::mbar_init(p_ready, 4);
    ptx::mbar_init(o_done, 1);
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *never_flag = 0;
    ptx::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmQ);
    ptx::prefetch_tmap(&tmC);
    ptx::prefetch_tmap(&tmKr);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && nchunk > 0) {
      ptx::mbar_arrive_expect_tx(q_full, kQBytes);
      for (int c = 0; c < 9; ++c) ptx::tma_load_2d(sQ + c * kQBox, &tmQ, q_full, c * 64, b * kHeads);
      // boxes in the order their previous readers finish: k_pe_rot (S^T), then the latent
      // boxes in O^T block order; box c of chunk j waits for its chunk j-1 readers
      int loaded[kBoxes] = {};  // loads issued per box
      bool ok = true;
      for (int j = 0; ok && j < nchunk; ++j) {
        const int y = row0 + t_begin + j * kChunk;
        for (int o = 0; o < kBoxes; ++o) {
          const int c = o == 0 ? 8 : o - 1;
          if (!ptx::mbar_wait(box_empty0 + 8u * c, (j & 1) ^ 1u, abort_flag, p.status,
                              kTimeoutCycles, DS_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          const uint32_t fb = box_full0 + 8u * c;
          ptx::mbar_arrive_expect_tx(fb, kBox);
          if (c < 8) ptx::tma_load_2d(sC + c * kBox, &tmC, fb, c * 64, y);
          else ptx::tma_load_2d(sC + c * kBox, &tmKr, fb, 0, y);
          ++loaded[c];
        }
      }
      // no copy may still be in flight when the CTA exits: the last load of each box
      ptx::mbar_wait(q_full, 0, never_flag, p.status, kTimeoutCycles, DS_ERR_TIMEOUT);
      for (int c = 0; c < kBoxes; ++c)
        if (loaded[c] > 0)
          ptx::mbar_wait(box_full0 + 8u * c, (loaded[c] - 1) & 1, never_flag, p.status,
                         kTimeoutCycles, DS_ERR_TIMEOUT);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && nchunk > 0) {
      constexpr uint32_t idesc_s = ptx::idesc_bf16_f32(128, kHeads);
      constexpr uint32_t idesc_o = ptx::idesc_bf16_f32_amn(128, kHeads);
      bool ok = ptx::mbar_wait(q_full, 0, abort_flag, p.status, kTimeoutCycles, DS_ERR_TIMEOUT);
      for (int j = 0; ok && j < nchunk; ++j) {
        // S2^T = K_rot Q_pe^T over the 64 RoPE columns, then S1^T = C Q'^T over the 512
        // latent ones, box by box as the boxes land
        for (int o = 0; o < kBoxes; ++o) {
          const int c = o == 0 ? 8 : o - 1;
          if (!ptx::mbar_wait(box_full0 + 8u * c, j & 1, abort_flag, p.status, kTimeoutCycles,
                              DS_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t cb = sC + c * kBox, qb = sQ + c * kQBox;
          const uint32_t d = tmem + (c == 8 ? kColS2 : kColS1);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            ptx::umma_f16(d, ptx::sw128_kmajor_desc(cb + kk * 32),
                          ptx::sw128_kmajor_desc(qb + kk * 32), idesc_s,
                          (kk > 0 || o > 1) ? 1u : 0u);
          if (c == 8) ptx::umma_commit(box_empty0 + 8u * 8);  // k_pe_rot: read only by S^T
        }
        if (!ok) break;
        ptx::umma_commit(s_full);
        if (!ptx::mbar_wait(p_ready, j & 1, abort_flag, p.status, kTimeoutCycles,
                            DS_ERR_TIMEOUT))
          break;
        ptx::tc_fence_after();
        // O^T (4 blocks of 128 latent dims) += C^T P^T: A = latent boxes 2i, 2i+1 read
        // MN-major (64 dims per 128-byte row, the next 64 one box = 16 KiB on; tokens 128
        // bytes apart), B = P^T [16 heads x 128 tokens] K-major (two 64-token atoms); the
        // two boxes go back to the producer as soon as the block's MMAs are done
#pragma unroll 1
        for (int i = 0; i < 4; ++i) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t a = sC + (2 * i) * kBox + kk * 16 * 128;
            const uint32_t pb = sP + (kk >> 2) * kQBox + (kk & 3) * 32;
            ptx::umma_f16(tmem + kColO + i * kHeads, ptx::sw128_mnmajor_desc(a, kBox),
                          ptx::sw128_kmajor_desc(pb), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
          }
          ptx::umma_commit(box_empty0 + 8u * (2 * i));
          ptx::umma_commit(box_empty0 + 8u * (2 * i + 1));
        }
        ptx::umma_commit(o_done);
      }
      ptx::umma_commit(drain_bar);
      ptx::mbar_wait(drain_bar, 0, never_flag, p.status, kTimeoutCycles, DS_ERR_TIMEOUT);
    }
  } else {
    // ------------------------------------------------------------------ softmax (warps 2-5)
    const int quarter = warp & 3;
    const int tl = quarter * 32 + lane;  // TMEM lane: token of S, latent dim of an O^T block
    const int tok = tl;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    constexpr float kLazy = 8.f;
    float m[kHeads], lsum[kHeads];
#pragma unroll
    for (int h = 0; h < kHeads; ++h) {
      m[h] = -INFINITY;
      lsum[h] = 0.f;
    }
    bool ok = nchunk > 0;
    for (int j = 0; ok && j < nchunk; ++j) {
      const int t = t_begin + j * kChunk + tok;
      const bool live = t < t_end;
      const float r = live ? __ldg(p.rstd + row0 + t) : 0.f;  // in flight during the wait
      int w_ok = 1;
      if (lane == 0)
        w_ok = ptx::mbar_wait(s_full, j & 1, abort_flag, p.status, kTimeoutCycles,
                              DS_ERR_TIMEOUT)
                   ? 1
                   : 0;
      w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
      // all four warps agree before the named barriers below (a lone early exit would
      // leave the others waiting in them)
      if (lane == 0) red[64 + quarter] = w_ok ? 0.f : 1.f;
      ptx::named_bar_sync(1, 128);
      const bool all_ok = red[64] == 0.f && red[65] == 0.f && red[66] == 0.f && red[67] == 0.f;
      ptx::named_bar_sync(1, 128);
      if (!all_ok) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      uint32_t s1[32];
      ptx::tmem_ld32(tmem + lane_off + kColS1, s1);  // columns 0..31: S1 (0..15), S2 (16..31)
      ptx::tmem_wait_ld(s1);
      float s[kHeads];
      float mx[kHeads];
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        s[h] = live ? (r * __uint_as_float(s1[h]) + __uint_as_float(s1[16 + h])) * p.scale_log2
                    : -INFINITY;
        mx[h] = s[h];
      }
#pragma unroll
      for (int h = 0; h < kHeads; ++h)
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], d));
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < kHeads; ++h) red[quarter * kHeads + h] = mx[h];
      }
      ptx::named_bar_sync(1, 128);
      float alpha[kHeads];
      bool any_rescale = false;
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        const float mc = fmaxf(fmaxf(red[h], red[kHeads + h]), fmaxf(red[2 * kHeads + h], red[3 * kHeads + h]));
        alpha[h] = 1.f;
        if (mc > m[h] + kLazy) {
          alpha[h] = ptx::ex2(m[h] - mc);  // 0 on the first chunk
          m[h] = mc;
          any_rescale = true;
        }
      }
      // P^T (times rstd) into the 16 x 128 shared tile: head h is row h of atom tok / 64,
      // token tok is element tok % 64 of the row's 128 bytes, 16-byte chunks XOR-swizzled
      // by (h & 7) as the SWIZZLE_128B operand layout expects
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        const float pv = ptx::ex2(s[h] - m[h]);  // 0 for a token that is not live
        lsum[h] = lsum[h] * alpha[h] + pv;
        {
          const int w = tok & 63;
          const uint32_t chunk = (static_cast<uint32_t>(w >> 3) ^ static_cast<uint32_t>(h & 7));
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(sPgen + (tok >> 6) * kQBox +
                                                                 h * 128 + chunk * 16) + (w & 7);
          *dst = __float2bfloat16_rn(pv * r);
        }
      }
      // the previous chunk's O^T MMAs must have landed before O^T is touched (o_done is
      // waited at every chunk, in order; the next O^T cannot start before this warp's
      // p_ready arrival, so the barrier is never more than one phase ahead)
      if (j > 0) {
        int o_ok = 1;
        if (lane == 0)
          o_ok = ptx::mbar_wait(o_done, (j - 1) & 1, abort_flag, p.status, kTimeoutCycles,
                                DS_ERR_TIMEOUT)
                     ? 1
                     : 0;
        if (!__shfl_sync(0xffffffffu, o_ok, 0)) ok = false;
        ptx::tc_fence_after();
        if (ok && any_rescale) {  // the same decision in every thread (shared maxima)
          uint32_t o[4][32];
          ptx::tmem_ld32(tmem + lane_off + kColO, o[0]);
          ptx::tmem_ld32(tmem + lane_off + kColO + 32, o[1]);
          ptx::tmem_wait_ld2(o[0], o[1]);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              o[c][i] = __float_as_uint(__uint_as_float(o[c][i]) * alpha[i & 15]);
            ptx::tmem_st32(tmem + lane_off + kColO + c * 32, o[c]);
          }
        }
      }
      ptx::tmem_wait_st();
      ptx::fence_async_shared();  // P^T stores -> visible to the tensor cores
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(p_ready);
      ptx::named_bar_sync(1, 128);  // red[] is rewritten by the next chunk
    }
    if (ok) {
      int o_ok = 1;
      if (lane == 0)
        o_ok = ptx::mbar_wait(o_done, (nchunk - 1) & 1, abort_flag, p.status, kTimeoutCycles,
                              DS_ERR_TIMEOUT)
                   ? 1
                   : 0;
      ok = __shfl_sync(0xffffffffu, o_ok, 0) != 0;
    }
    // per-head sums over the 128 tokens of all chunks: shuffles, then the four warps
#pragma unroll
    for (int h = 0; h < kHeads; ++h)
#pragma unroll
      for (int d = 16; d > 0; d >>= 1) lsum[h] += __shfl_xor_sync(0xffffffffu, lsum[h], d);
    ptx::named_bar_sync(1, 128);
    if (lane == 0) {
#pragma unroll
      for (int h = 0; h < kHeads; ++h) red[quarter * kHeads + h] = lsum[h];
    }
    ptx::named_bar_sync(1, 128);
    float* ml = p.part_ml + (static_cast<int64_t>(b) * p.nsplit + split) * 2 * kHeads;
    if (threadIdx.x == 64) {  // warp 2 lane 0
      for (int h = 0; h < kHeads; ++h) {
        ml[h] = (ok && nchunk > 0) ? m[h] : -INFINITY;
        ml[kHeads + h] = (ok && nchunk > 0)
                             ? red[h] + red[kHeads + h] + red[2 * kHeads + h] + red[3 * kHeads + h]
                             : 0.f;
      }
    }
    float* po = p.part_o + (static_cast<int64_t>(b) * p.nsplit + split) * kHeads * kLatent;
    if (ok && nchunk > 0) {
      ptx::tc_fence_after();
      uint32_t o[2][32];
      ptx::tmem_ld32(tmem + lane_off + kColO, o[0]);
      ptx::tmem_ld32(tmem + lane_off + kColO + 32, o[1]);
      ptx::tmem_wait_ld2(o[0], o[1]);
      // lane tl of block i holds latent dim i*128 + tl for the 16 heads
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int h = 0; h < kHeads; ++h)
          po[h * kLatent + i * 128 + tl] = __uint_as_float(o[i >> 1][(i & 1) * 16 + h]);
    } else {
      for (int i = 0; i < 4; ++i)
        for (int h = 0; h < kHeads; ++h) po[h * kLatent + i * 128 + tl] = 0.f;
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

// Merge the splits of each (sequence, head): o_lat = sum_s 2^(m_s - M) o_s / sum_s 2^(m_s - M) l_s
// -> bf16 out[b, h*512 + d].
__global__ void __launch_bounds__(128)
    mla_decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                              int nsplit, __nv_bfloat16* __restrict__ out) {
  const int b = blockIdx.x / kHeads, h = blockIdx.x - (blockIdx.x / kHeads) * kHeads;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s)
    M = fmaxf(M, __ldg(part_ml + (static_cast<int64_t>(b) * nsplit + s) * 2 * kHeads + h));
  float L = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < nsplit; ++s) {
    const float* ml = part_ml + (static_cast<int64_t>(b) * nsplit + s) * 2 * kHeads;
    const float ms = __ldg(ml + h);
    if (ms == -INFINITY) continue;
    const float w = ptx::ex2(ms - M);
    L += w * __ldg(ml + kHeads + h);
    const float* po = part_o + ((static_cast<int64_t>(b) * nsplit + s) * kHeads + h) * kLatent;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] += w * __ldg(po + k * 128 + threadIdx.x);
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  __nv_bfloat16* o = out + (static_cast<int64_t>(b) * kHeads + h) * kLatent;
#pragma unroll
  for (int k = 0; k < 4; ++k) o[k * 128 + threadIdx.x] = __float2bfloat16_rn(acc[k] * inv);
}

// Cache append: for n_new tokens of each of `batch` sequences at positions pos0 ..: token i
// of sequence b reads its latent from src_lat + (b*src_bstride + i)*lat_ld and its raw k_pe
// from src_kpe + (b*src_bstride + i)*kpe_ld; the raw values go into the cache (unless
// copy_raw is 0: the side arrays of tokens already in the cache are being refreshed),
// rstd = rsqrt(mean(latent^2) + eps) and k_pe rotated at its position (the interleave ->
// half RoPE of src/reference/mla.py:176-206) into the side arrays.  One warp per token.
__global__ void __launch_bounds__(256)
    cache_append_kernel(const __nv_bfloat16* __restrict__ src_lat, int lat_ld,
                        const __nv_bfloat16* __restrict__ src_kpe, int kpe_ld, int src_bstride,
                        int batch, int n_new, int pos0, const int* pos0_dev, int max_seq,
                        int copy_raw,
                        __nv_bfloat16* c_lat, __nv_bfloat16* c_kpe, float* __restrict__ c_rstd,
                        __nv_bfloat16* __restrict__ c_kpe_rot,
                        const __nv_bfloat16* __restrict__ cos_t,
                        const __nv_bfloat16* __restrict__ sin_t, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t w = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  if (w >= static_cast<int64_t>(batch) * n_new) return;
  const int b = static_cast<int>(w / n_new), i = static_cast<int>(w - static_cast<int64_t>(b) * n_new);
  const int pos = (pos0_dev != nullptr ? *pos0_dev : pos0) + i;
  const int64_t srow = static_cast<int64_t>(b) * src_bstride + i;
  const int64_t dst = static_cast<int64_t>(b) * max_seq + pos;
  // latent: 512 = 32 lanes x 16 elements
  const uint4* l4 = reinterpret_cast<const uint4*>(src_lat + srow * lat_ld) + 2 * lane;
  const uint4 a0 = l4[0], a1 = l4[1];
  const __nv_bfloat16* kp = src_kpe + srow * kpe_ld;
  uint4 kraw = make_uint4(0, 0, 0, 0);
  if (lane < 8) kraw = reinterpret_cast<const uint4*>(kp)[lane];
  const float xa = __bfloat162float(kp[2 * lane]), xb = __bfloat162float(kp[2 * lane + 1]);
  __syncwarp();  // every read of the source (it may be the cache itself) before any write
  if (copy_raw) {
    uint4* d4 = reinterpret_cast<uint4*>(c_lat + dst * kLatent) + 2 * lane;
    d4[0] = a0;
    d4[1] = a1;
    if (lane < 8) reinterpret_cast<uint4*>(c_kpe + dst * kRope)[lane] = kraw;
  }
  float ss = 0.f;
  const __nv_bfloat16* e0 = reinterpret_cast<const __nv_bfloat16*>(&a0);
  const __nv_bfloat16* e1 = reinterpret_cast<const __nv_bfloat16*>(&a1);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float x0 = __bfloat162float(e0[k]), x1 = __bfloat162float(e1[k]);
    ss = fmaf(x0, x0, fmaf(x1, x1, ss));
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
  if (lane == 0) c_rstd[dst] = rsqrtf(ss / kLatent + eps);
  // k_pe: 32 rotation pairs, one per lane
  const __nv_bfloat16* cr = cos_t + static_cast<int64_t>(pos) * kRope;
  const __nv_bfloat16* sr = sin_t + static_cast<int64_t>(pos) * kRope;
  __nv_bfloat16* kr = c_kpe_rot + dst * kRope;
  kr[lane] = __float2bfloat16_rn(xa * __bfloat162float(cr[lane]) - xb * __bfloat162float(sr[lane]));
  kr[32 + lane] =
      __float2bfloat16_rn(xb * __bfloat162float(cr[32 + lane]) + xa * __bfloat162float(sr[32 + lane]));
}

// Decode query: Q[b, h] = [q'_h (512, copied) | rope(q_pe_h) at position pos (64)] from the
// projection row of sequence b.  One warp per (sequence, head).
__global__ void __launch_bounds__(256)
    decode_q_kernel(const __nv_bfloat16* __restrict__ proj, int ld, int qpe_col, int batch,
                    int heads, int pos_host, const int* pos_dev,
                    const __nv_bfloat16* __restrict__ cos_t,
                    const __nv_bfloat16* __restrict__ sin_t, __nv_bfloat16* __restrict__ q) {
  const int lane = threadIdx.x & 31;
  const int64_t w = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  if (w >= static_cast<int64_t>(batch) * heads) return;
  const int b = static_cast<int>(w / heads), h = static_cast<int>(w - static_cast<int64_t>(b) * heads);
  const int pos = pos_dev != nullptr ? *pos_dev : pos_host;
  const __nv_bfloat16* row = proj + static_cast<int64_t>(b) * ld;
  __nv_bfloat16* dst = q + w * kQCols;
  const uint4* s4 = reinterpret_cast<const uint4*>(row + h * kLatent) + 2 * lane;
  uint4* d4 = reinterpret_cast<uint4*>(dst) + 2 * lane;
  d4[0] = s4[0];
  d4[1] = s4[1];
  const __nv_bfloat16* qp = row + qpe_col + h * kRope;
  const float xa = __bfloat162float(qp[2 * lane]), xb = __bfloat162float(qp[2 * lane + 1]);
  const __nv_bfloat16* cr = cos_t + static_cast<int64_t>(pos) * kRope;
  const __nv_bfloat16* sr = sin_t + static_cast<int64_t>(pos) * kRope;
  dst[kLatent + lane] =
      __float2bfloat16_rn(xa * __bfloat162float(cr[lane]) - xb * __bfloat162float(sr[lane]));
  dst[kLatent + 32 + lane] =
      __float2bfloat16_rn(xb * __bfloat162float(cr[32 + lane]) + xa * __bfloat162float(sr[32 + lane]));
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
bool g_attr_set[64] = {};
std::mutex g_attr_mutex;

int tmap_2d(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, uint32_t box_rows) {
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
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  cuuint32_t box[2] = {64u, box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  const CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DS_OK;
}

int nsplit_for(int batch, int len, int num_sms, int* chunks_per_split) {
  const int chunks = (len + kChunk - 1) / kChunk;
  // one wave of one CTA per SM, at least one chunk per split
  int want = num_sms / batch;
  if (want > chunks) want = chunks;
  if (want < 1) want = 1;
  *chunks_per_split = (chunks + want - 1) / want;
  return (chunks + *chunks_per_split - 1) / *chunks_per_split;
}

}  // namespace

// The cache's device-side length += n (one thread), after the step's kernels have used it.
__global__ void len_add_kernel(int* len, int n) { *len += n; }

int launch_cache_append(const void* src_lat, int lat_ld, const void* src_kpe, int kpe_ld,
                        int src_bstride, int batch, int n_new, int pos0, const int* pos0_dev,
                        int max_seq, int copy_raw, void* c_lat, void* c_kpe, float* c_rstd,
                        void* c_kpe_rot, const void* cos_t, const void* sin_t, float eps,
                        cudaStream_t s) {
  const int64_t warps = static_cast<int64_t>(batch) * n_new;
  if (warps == 0) return DS_OK;
  cache_append_kernel<<<static_cast<int>((warps * 32 + 255) / 256), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(src_lat), lat_ld,
      static_cast<const __nv_bfloat16*>(src_kpe), kpe_ld, src_bstride, batch, n_new, pos0,
      pos0_dev, max_seq, copy_raw, static_cast<__nv_bfloat16*>(c_lat), static_cast<__nv_bfloat16*>(c_kpe),
      c_rstd, static_cast<__nv_bfloat16*>(c_kpe_rot), static_cast<const __nv_bfloat16*>(cos_t),
      static_cast<const __nv_bfloat16*>(sin_t), eps);
  DS_LAUNCH_CHECK("cache_append_kernel");
  return DS_OK;
}

size_t attn_workspace(int batch, int len, int num_sms) {
  int cps = 1;
  const int ns = nsplit_for(batch, len, num_sms, &cps);
  return align_up(static_cast<size_t>(batch) * ns * kHeads * kLatent * 4, 256) +
         align_up(static_cast<size_t>(batch) * ns * 2 * kHeads * 4, 256);
}

// Attention of one new token per sequence over positions [0, len) of the cache; q: [batch*16,
// 576] bf16; out: o_lat [batch, 16*512] bf16.
int launch_decode_attention(const void* q, const void* c_lat, const float* c_rstd,
                            const void* c_kpe_rot, int batch, int max_seq, int len,
                            const int* len_dev, float softmax_scale, void* out, void* workspace,
                            size_t ws_bytes, cudaStream_t s) {
  DeviceInfo di;
  DS_TRY(device_info(&di));
  int cps = 1;
  // with the length on the device the splits cover max_seq; splits past the length exit
  const int ns = nsplit_for(batch, len_dev != nullptr ? max_seq : len, di.num_sms, &cps);
  DS_REQUIRE(ws_bytes >= attn_workspace(batch, len_dev != nullptr ? max_seq : len, di.num_sms),
             "decode attention: workspace");
  {
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    if (!g_attr_set[di.device]) {
      DS_CUDA(cudaFuncSetAttribute(mla_decode_attn_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(kSmemBytes)));
      g_attr_set[di.device] = true;
    }
  }
  CUtensorMap tq, tc, tk;
  DS_TRY(tmap_2d(&tq, q, static_cast<int64_t>(batch) * kHeads, kQCols, 16u));
  DS_TRY(tmap_2d(&tc, c_lat, static_cast<int64_t>(batch) * max_seq, kLatent, kChunk));
  DS_TRY(tmap_2d(&tk, c_kpe_rot, static_cast<int64_t>(batch) * max_seq, kRope, kChunk));
  Params p{};
  p.batch = batch;
  p.max_seq = max_seq;
  p.len = len;
  p.len_dev = len_dev;
  p.nsplit = ns;
  p.chunks_per_split = cps;
  p.rstd = c_rstd;
  p.scale_log2 = static_cast<float>(static_cast<double>(softmax_scale) * 1.4426950408889634);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  p.part_o = reinterpret_cast<float*>(w);
  p.part_ml = reinterpret_cast<float*>(
      w + align_up(static_cast<size_t>(batch) * ns * kHeads * kLatent * 4, 256));
  p.status = device_status_ptr();
  if (p.status == nullptr) return fail(DS_ERR_CUDA, "device status word unavailable");
  mla_decode_attn_kernel<<<batch * ns, kThreads, kSmemBytes, s>>>(tq, tc, tk, p);
  DS_LAUNCH_CHECK("mla_decode_attn_kernel");
  mla_decode_combine_kernel<<<batch * kHeads, 128, 0, s>>>(p.part_o, p.part_ml, ns,
                                                           static_cast<__nv_bfloat16*>(out));
  DS_LAUNCH_CHECK("mla_decode_combine_kernel");
  return DS_OK;
}

int launch_decode_q(const void* proj, int ld, int qpe_col, int batch, int heads, int pos,
                    const int* pos_dev, const void* cos_t, const void* sin_t, void* q,
                    cudaStream_t s) {
  const int64_t warps = static_cast<int64_t>(batch) * heads;
  decode_q_kernel<<<static_cast<int>((warps * 32 + 255) / 256), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(proj), ld, qpe_col, batch, heads, pos, pos_dev,
      static_cast<const __nv_bfloat16*>(cos_t), static_cast<const __nv_bfloat16*>(sin_t),
      static_cast<__nv_bfloat16*>(q));
  DS_LAUNCH_CHECK("decode_q_kernel");
  return DS_OK;
}

}  // namespace dec
}  // namespace ds

// ---- C ABI ------------------------------------------------------------------------------------
namespace {

constexpr int kDecHeads = 16;

int dec_proj_cols(int heads) { return heads * 512 + heads * 64 + 512 + 64; }

struct DecBuffers {
  void* proj;      // bf16 [batch, dec_proj_cols]
  void* q;         // bf16 [batch*16, 576]
  void* olat;      // bf16 [batch, 16*512]
  void* attn;      // f32 attention partials
  float* partial;  // f32 split-K partials of the two projections
};

ds::gemm::Problem dense(const void* A, int64_t rows, int K, const void* B, int N, void* out);

// the decode step's projections: x [batch, hidden] -> proj, and o_lat -> out; with 64 rows
// their output tiles leave most SMs idle, so they run split-K
size_t dec_partial_bytes(int batch, int hidden, int num_sms) {
  ds::gemm::Problem a = dense(nullptr, batch, hidden, nullptr, dec_proj_cols(kDecHeads), nullptr);
  ds::gemm::Problem o = dense(nullptr, batch, kDecHeads * 512, nullptr, hidden, nullptr);
  const size_t pa = ds::gemm::partial_bytes(a, ds::gemm::choose_k_splits(a, num_sms));
  const size_t po = ds::gemm::partial_bytes(o, ds::gemm::choose_k_splits(o, num_sms));
  return pa > po ? pa : po;
}

size_t carve_dec(ds::Carve& c, DecBuffers* b, int batch, int max_seq, int hidden, int num_sms) {
  DecBuffers x{};
  x.proj = c.take<__nv_bfloat16>(static_cast<size_t>(batch) * dec_proj_cols(kDecHeads));
  x.q = c.take<__nv_bfloat16>(static_cast<size_t>(batch) * kDecHeads * 576);
  x.olat = c.take<__nv_bfloat16>(static_cast<size_t>(batch) * kDecHeads * 512);
  const size_t aw = ds::dec::attn_workspace(batch, max_seq, num_sms);
  x.attn = c.take<uint8_t>(aw);
  x.partial = c.take<float>(dec_partial_bytes(batch, hidden, num_sms) / sizeof(float));
  if (b) *b = x;
  return ds::align_up(c.used, 256);
}

// a dense problem; `partial` set: split-K when the output tiles leave most SMs idle
ds::gemm::Problem dense_split(const void* A, int64_t rows, int K, const void* B, int N, void* out,
                              float* partial, int num_sms) {
  ds::gemm::Problem p = dense(A, rows, K, B, N, out);
  p.k_splits = ds::gemm::choose_k_splits(p, num_sms);
  p.partial = partial;
  return p;
}

ds::gemm::Problem dense(const void* A, int64_t rows, int K, const void* B, int N, void* out) {
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

int ds_mla_cache_append(const void* latent_bf16, int latent_ld, const void* kpe_bf16, int kpe_ld,
                        int src_rows_per_seq, int batch, int new_tokens, int pos0, int max_seq,
                        int copy_raw, void* cache_latent_bf16, void* cache_kpe_bf16,
                        float* cache_rstd, void* cache_kpe_rot_bf16, const void* cos_bf16,
                        const void* sin_bf16, float eps, void* stream) {
  DS_REQUIRE(batch >= 0 && new_tokens >= 0 && pos0 >= 0, "mla_cache_append: bad shape");
  DS_REQUIRE(pos0 + new_tokens <= max_seq, "mla_cache_append: cache overflow");
  if (batch == 0 || new_tokens == 0) return DS_OK;
  DS_REQUIRE(latent_bf16 && kpe_bf16 && cache_latent_bf16 && cache_kpe_bf16 && cache_rstd &&
                 cache_kpe_rot_bf16 && cos_bf16 && sin_bf16,
             "mla_cache_append: null pointer");
  DS_REQUIRE(latent_ld % 8 == 0 && kpe_ld % 8 == 0 && ds::aligned16(latent_bf16) &&
                 ds::aligned16(kpe_bf16),
             "mla_cache_append: rows must start on 16-byte boundaries");
  return ds::dec::launch_cache_append(latent_bf16, latent_ld, kpe_bf16, kpe_ld, src_rows_per_seq,
                                      batch, new_tokens, pos0, nullptr, max_seq, copy_raw,
                                      cache_latent_bf16, cache_kpe_bf16, cache_rstd,
                                      cache_kpe_rot_bf16, cos_bf16, sin_bf16, eps,
                                      static_cast<cudaStream_t>(stream));
}

size_t ds_mla_decode_workspace_size(int batch, int max_seq, int hidden) {
  ds::DeviceInfo di;
  if (ds::device_info(&di) != DS_OK) return 0;
  ds::Carve c(nullptr, 0);
  return carve_dec(c, nullptr, batch, max_seq, hidden, di.num_sms);
}

int ds_mla_decode_step(const void* x_bf16, const void* w_dec_bf16, const void* w_out_bf16,
                       const void* cos_bf16, const void* sin_bf16, void* cache_latent_bf16,
                       void* cache_kpe_bf16, float* cache_rstd, void* cache_kpe_rot_bf16,
                       int batch, int max_seq, int cache_len, int32_t* cache_len_dev, int hidden,
                       int heads, float eps, float softmax_scale, void* out_bf16,
                       void* workspace, size_t workspace_bytes, void** events, void* stream) {
  DS_REQUIRE(batch >= 0 && hidden > 0 && hidden % 8 == 0, "mla_decode_step: bad shape");
  DS_REQUIRE(heads == kDecHeads, "mla_decode_step: %d heads (the decode kernel serves 16)", heads);
  DS_REQUIRE(cache_len >= 0 && cache_len < max_seq, "mla_decode_step: cache is full");
  if (batch == 0) return DS_OK;
  DS_REQUIRE(x_bf16 && w_dec_bf16 && w_out_bf16 && cos_bf16 && sin_bf16 && cache_latent_bf16 &&
                 cache_kpe_bf16 && cache_rstd && cache_kpe_rot_bf16 && out_bf16 && workspace,
             "mla_decode_step: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto mark = [&](int i) -> int {
    if (events != nullptr && events[i] != nullptr)
      DS_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[i]), s));
    return DS_OK;
  };
  ds::DeviceInfo di;
  DS_TRY(ds::device_info(&di));
  ds::Carve c(workspace, workspace_bytes);
  DecBuffers b;
  carve_dec(c, &b, batch, max_seq, hidden, di.num_sms);
  if (!c.ok()) return ds::fail(DS_ERR_WORKSPACE, "mla_decode_step: workspace needs %zu bytes", c.used);
  const int P = dec_proj_cols(heads);
  const int qpe_col = heads * 512, lat_col = qpe_col + heads * 64, kpe_col = lat_col + 512;
  DS_TRY(mark(0));
  DS_TRY(ds::gemm::launch(
      dense_split(x_bf16, batch, hidden, w_dec_bf16, P, b.proj, b.partial, di.num_sms), s));
  DS_TRY(mark(1));
  DS_TRY(ds::dec::launch_cache_append(static_cast<const __nv_bfloat16*>(b.proj) + lat_col, P,
                                      static_cast<const __nv_bfloat16*>(b.proj) + kpe_col, P, 1,
                                      batch, 1, cache_len, cache_len_dev, max_seq, 1,
                                      cache_latent_bf16,
                                      cache_kpe_bf16, cache_rstd, cache_kpe_rot_bf16, cos_bf16,
                                      sin_bf16, eps, s));
  DS_TRY(ds::dec::launch_decode_q(b.proj, P, qpe_col, batch, heads, cache_len, cache_len_dev,
                                  cos_bf16, sin_bf16, b.q, s));
  DS_TRY(mark(2));
  DS_TRY(ds::dec::launch_decode_attention(b.q, cache_latent_bf16, cache_rstd, cache_kpe_rot_bf16,
                                          batch, max_seq, cache_len + 1, cache_len_dev,
                                          softmax_scale, b.olat, b.attn,
                                          ds::dec::attn_workspace(batch, max_seq, di.num_sms), s));
  if (cache_len_dev != nullptr) {
    ds::dec::len_add_kernel<<<1, 1, 0, s>>>(cache_len_dev, 1);
    DS_LAUNCH_CHECK("len_add_kernel");
  }
  DS_TRY(mark(3));
  DS_TRY(ds::gemm::launch(dense_split(b.olat, batch, heads * 512, w_out_bf16, hidden, out_bf16,
                                      b.partial, di.num_sms),
                          s));
  DS_TRY(mark(4));
  return DS_OK;
}

}  // extern "C"

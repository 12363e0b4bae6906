// MLA projection-path bandwidth kernels: RMSNorm over the 512-d kv latent (K8) and RoPE on
// the 64-d rope slices of q and k (K10), with their C-ABI entry points.
//
// RMSNorm follows src/reference/mla.py:59-64 (f32 statistics) with the single rounding of
// src/kernels/mla/rms_norm.cu:104-114; RoPE implements the interleave->half rotation of
// src/reference/mla.py:183-206 in the per-element form of src/kernels/mla/rope.cu:23-26.
#include <mutex>

#include "kernels.cuh"
#include "ptx.cuh"

namespace ds {
namespace {

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 f32x8_to_bf16(const float (&f)[8]) {
  uint4 r;
  uint32_t* u = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    u[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  return r;
}

// Contiguous rows of at most 512 elements (the 512-d kv latent): a pipelined ring.  Each CTA
// walks tiles of kNormTileRows rows; thread 0 keeps kNormStages tiles in flight with one bulk
// copy each (global -> shared, no registers spent on the bytes in flight) while the 8 warps
// normalise the oldest tile from shared memory (2 rows per warp, f32 statistics, weights held
// in registers) and write it with 16-byte stores; the stage is refilled once every warp has
// read it.  DRAM latency is paid once per CTA, not once per tile.  Every wait is bounded: on
// expiry the CTA records DS_ERR_TIMEOUT, waits (bounded) for its copies in flight, returns.
constexpr int kNormTileRows = 16;
constexpr int kNormStages = 4;
__global__ void __launch_bounds__(256)
    rms_norm_ring_kernel(const __nv_bfloat16* __restrict__ in, const float4* __restrict__ weight,
                         uint4* __restrict__ out, int rows, int H, float eps, int* status,
                         long long timeout_cycles) {
  extern __shared__ __align__(128) uint8_t ring[];  // kNormStages x kNormTileRows x H bf16
  __shared__ __align__(8) uint64_t bars[kNormStages];
  __shared__ int abort_flag;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ntiles = (rows + kNormTileRows - 1) / kNormTileRows;
  const int mine = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const uint32_t stage_bytes = static_cast<uint32_t>(kNormTileRows) * H * 2;
  const uint32_t ring0 = ptx::smem_u32(ring);
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int st = 0; st < kNormStages; ++st) ptx::mbar_init(ptx::smem_u32(&bars[st]), 1);
    ptx::fence_barrier_init();
  }
  __syncthreads();
  auto issue = [&](int i) {  // thread 0: the CTA's i-th tile into stage i % kNormStages
    const int tile = blockIdx.x + i * gridDim.x;
    const int r0 = tile * kNormTileRows;
    const uint32_t bytes = static_cast<uint32_t>(min(kNormTileRows, rows - r0)) * H * 2;
    const uint32_t bar = ptx::smem_u32(&bars[i % kNormStages]);
    ptx::mbar_arrive_expect_tx(bar, bytes);
    ptx::bulk_load_1d(ring0 + (i % kNormStages) * stage_bytes, in + static_cast<int64_t>(r0) * H,
                      bytes, bar);
  };
  int issued = 0;
  if (threadIdx.x == 0)
    for (; issued < min(mine, kNormStages); ++issued) issue(issued);
  const int H8 = H >> 3;
  float wv[2][8];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int c = u * 32 + lane;
    if (c < H8) {
      const float4 w0 = __ldg(weight + 2 * c), w1 = __ldg(weight + 2 * c + 1);
      wv[u][0] = w0.x; wv[u][1] = w0.y; wv[u][2] = w0.z; wv[u][3] = w0.w;
      wv[u][4] = w1.x; wv[u][5] = w1.y; wv[u][6] = w1.z; wv[u][7] = w1.w;
    }
  }
  const float inv_h = 1.f / static_cast<float>(H);
  int done = 0;
  for (; done < mine; ++done) {
    const int st = done % kNormStages;
    if (!ptx::mbar_wait(ptx::smem_u32(&bars[st]), (done / kNormStages) & 1, &abort_flag, status,
                        timeout_cycles, DS_ERR_TIMEOUT))
      break;
    const int r0 = (blockIdx.x + done * gridDim.x) * kNormTileRows;
    const int nrows = min(kNormTileRows, rows - r0);
    const uint4* t4 = reinterpret_cast<const uint4*>(ring + st * stage_bytes);
    uint4 v[2][2];
    float ss[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int r = warp * 2 + j;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = u * 32 + lane;
        if (r < nrows && c < H8) {
          v[j][u] = t4[r * H8 + c];
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[j][u]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            ss[j] = fmaf(f.x, f.x, ss[j]);
            ss[j] = fmaf(f.y, f.y, ss[j]);
          }
        }
      }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      ss[0] += __shfl_xor_sync(0xffffffffu, ss[0], d);
      ss[1] += __shfl_xor_sync(0xffffffffu, ss[1], d);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int r = warp * 2 + j;
      if (r >= nrows) continue;
      const float scale = rsqrtf(ss[j] * inv_h + eps);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = u * 32 + lane;
        if (c >= H8) continue;
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[j][u]);
        uint4 o;
        uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h[i]);
          const __nv_bfloat162 bb =
              __floats2bfloat162_rn(f.x * scale * wv[u][2 * i], f.y * scale * wv[u][2 * i + 1]);
          ou[i] = *reinterpret_cast<const uint32_t*>(&bb);
        }
        out[static_cast<int64_t>(r0 + r) * H8 + c] = o;
      }
    }
    __syncthreads();  // every warp has read the stage: refill it
    if (threadIdx.x == 0 && issued < mine) issue(issued++);
  }
  if (done < mine && threadIdx.x == 0) {  // aborted: let the copies still in flight land
    int never = 0;
    for (int i = done; i < issued; ++i)
      ptx::mbar_wait(ptx::smem_u32(&bars[i % kNormStages]), (i / kNormStages) & 1, &never,
                     status, timeout_cycles, DS_ERR_TIMEOUT);
  }
}

// Decoder-layer glue (src/reference/decoder_layer.py:123-139 around RMSNorm,
// src/reference/mla.py:59-64): sum = bf16(residual + x), normed = bf16(w * sum * rsqrt(
// mean(sum^2) + eps)) with f32 statistics over the rounded sum; both written.  One warp per
// row of up to 2048 elements, both input rows' 16-byte loads issued before the math.
__global__ void __launch_bounds__(256)
    rms_norm_residual_kernel(const uint4* __restrict__ x, const uint4* __restrict__ res,
                             const float4* __restrict__ weight, uint4* __restrict__ sum_out,
                             uint4* __restrict__ normed, int rows, int H, float eps) {
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int H8 = H >> 3;
  const float inv_h = 1.f / static_cast<float>(H);
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const int64_t base = static_cast<int64_t>(r) * H8;
    uint4 a[8], b[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int c = u * 32 + lane;
      if (c < H8) {
        a[u] = __ldg(x + base + c);
        b[u] = __ldg(res + base + c);
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int c = u * 32 + lane;
      if (c >= H8) continue;
      float fa[8], fb[8];
      bf16x8_to_f32(a[u], fa);
      bf16x8_to_f32(b[u], fb);
      float sm[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sm[i] = fb[i] + fa[i];
      a[u] = f32x8_to_bf16(sm);  // the rounded sum: written out and normalised
      float fs[8];
      bf16x8_to_f32(a[u], fs);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(fs[i], fs[i], ss);
      sum_out[base + c] = a[u];
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
    const float scale = rsqrtf(ss * inv_h + eps);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int c = u * 32 + lane;
      if (c >= H8) continue;
      const float4 w0 = __ldg(weight + 2 * c), w1 = __ldg(weight + 2 * c + 1);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      float fs[8], o[8];
      bf16x8_to_f32(a[u], fs);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = fs[i] * scale * wv[i];
      normed[base + c] = f32x8_to_bf16(o);
    }
  }
}

// Rows of at most 512 elements (the 512-d kv latent): one warp takes two rows at a time and
// issues all four 16-byte loads per lane before the reductions, so twice the bytes are in
// flight per warp as with one row.
__global__ void __launch_bounds__(256)
    rms_norm_pair_kernel(const uint4* __restrict__ in, int64_t in_stride8,
                         const float4* __restrict__ weight, uint4* __restrict__ out,
                         int64_t out_stride8, int rows, int H, float eps) {
  const int lane = threadIdx.x & 31;
  const int H8 = H >> 3;
  const int warps = gridDim.x * (blockDim.x >> 5);
  const float inv_h = 1.f / static_cast<float>(H);
  for (int r0 = 2 * (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)); r0 < rows;
       r0 += 2 * warps) {
    uint4 v[2][2];
    float ss[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = u * 32 + lane;
        if (r0 + j < rows && c < H8) v[j][u] = __ldg(in + (r0 + j) * in_stride8 + c);
      }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = u * 32 + lane;
        if (r0 + j < rows && c < H8) {
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[j][u]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            ss[j] = fmaf(f.x, f.x, ss[j]);
            ss[j] = fmaf(f.y, f.y, ss[j]);
          }
        }
      }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      ss[0] += __shfl_xor_sync(0xffffffffu, ss[0], d);
      ss[1] += __shfl_xor_sync(0xffffffffu, ss[1], d);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float scale = rsqrtf(ss[j] * inv_h + eps);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = u * 32 + lane;
        if (r0 + j < rows && c < H8) {
          const float4 w0 = __ldg(weight + 2 * c);
          const float4 w1 = __ldg(weight + 2 * c + 1);
          const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[j][u]);
          uint4 o;
          uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            const __nv_bfloat162 b =
                __floats2bfloat162_rn(f.x * scale * wv[2 * i], f.y * scale * wv[2 * i + 1]);
            ou[i] = *reinterpret_cast<const uint32_t*>(&b);
          }
          out[(r0 + j) * out_stride8 + c] = o;
        }
      }
    }
  }
}

// One warp per row.  Rows of up to 2048 elements stay in registers (8 x 16 B per lane);
// longer rows take a second pass over global memory.
__global__ void __launch_bounds__(256)
    rms_norm_kernel(const __nv_bfloat16* __restrict__ in, int64_t in_stride,
                    const float* __restrict__ weight, __nv_bfloat16* __restrict__ out,
                    int64_t out_stride, int rows, int H, float eps, int vec_ok) {
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  const float inv_h = 1.f / static_cast<float>(H);
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const __nv_bfloat16* x = in + static_cast<int64_t>(r) * in_stride;
    __nv_bfloat16* y = out + static_cast<int64_t>(r) * out_stride;
    if (vec_ok && H <= 2048) {
      const int H8 = H >> 3;
      uint4 v[8];
      float ss = 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = u * 32 + lane;
        if (c < H8) {
          v[u] = __ldg(reinterpret_cast<const uint4*>(x) + c);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[u]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            ss = fmaf(f.x, f.x, ss);
            ss = fmaf(f.y, f.y, ss);
          }
        }
      }
#pragma unroll
      for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
      const float scale = rsqrtf(ss * inv_h + eps);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = u * 32 + lane;
        if (c < H8) {
          const float4 w0 = __ldg(reinterpret_cast<const float4*>(weight) + 2 * c);
          const float4 w1 = __ldg(reinterpret_cast<const float4*>(weight) + 2 * c + 1);
          const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[u]);
          uint4 o;
          uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            const __nv_bfloat162 b =
                __floats2bfloat162_rn(f.x * scale * wv[2 * i], f.y * scale * wv[2 * i + 1]);
            ou[i] = *reinterpret_cast<const uint32_t*>(&b);
          }
          reinterpret_cast<uint4*>(y)[c] = o;
        }
      }
    } else {
      const int H2 = H >> 1;
      const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(x);
      float ss = 0.f;
      for (int c = lane; c < H2; c += 32) {
        const float2 f = __bfloat1622float2(x2[c]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
#pragma unroll
      for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
      const float scale = rsqrtf(ss * inv_h + eps);
      __nv_bfloat162* y2 = reinterpret_cast<__nv_bfloat162*>(y);
      for (int c = lane; c < H2; c += 32) {
        const float2 f = __bfloat1622float2(x2[c]);
        y2[c] = __floats2bfloat162_rn(f.x * scale * weight[2 * c], f.y * scale * weight[2 * c + 1]);
      }
    }
  }
}

// One thread per 8 input elements (4 rotation pairs) of a row; q rows then k rows.
// cos/sin rows are shared by every head of a (batch, position).
__global__ void __launch_bounds__(256)
    rope_vec_kernel(const uint4* __restrict__ q, const uint4* __restrict__ k,
                    const __nv_bfloat16* __restrict__ cos_t, const __nv_bfloat16* __restrict__ sin_t,
                    uint4* __restrict__ qo, uint4* __restrict__ ko, int64_t q_rows,
                    int64_t k_rows, int heads, int seq, int D) {
  const int D8 = D >> 3, half = D >> 1;
  const int64_t total = (q_rows + k_rows) * D8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / D8;
    const int c = static_cast<int>(i - row * D8);
    const bool is_q = row < q_rows;
    const int64_t lrow = is_q ? row : row - q_rows;
    // (b, h, s) for q rows, (b, s) for k rows -> cos/sin row b*seq + s
    int64_t cs_row;
    if (is_q) {
      const int64_t s_ = lrow % seq;
      const int64_t b_ = lrow / (static_cast<int64_t>(seq) * heads);
      cs_row = b_ * seq + s_;
    } else {
      cs_row = lrow;
    }
    const uint4 xv = __ldg((is_q ? q : k) + lrow * D8 + c);
    const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&xv);
    const __nv_bfloat16* cr = cos_t + cs_row * D;
    const __nv_bfloat16* sr = sin_t + cs_row * D;
    const uint2 c_lo = __ldg(reinterpret_cast<const uint2*>(cr + 4 * c));
    const uint2 c_hi = __ldg(reinterpret_cast<const uint2*>(cr + half + 4 * c));
    const uint2 s_lo = __ldg(reinterpret_cast<const uint2*>(sr + 4 * c));
    const uint2 s_hi = __ldg(reinterpret_cast<const uint2*>(sr + half + 4 * c));
    const __nv_bfloat162* clo = reinterpret_cast<const __nv_bfloat162*>(&c_lo);
    const __nv_bfloat162* chi = reinterpret_cast<const __nv_bfloat162*>(&c_hi);
    const __nv_bfloat162* slo = reinterpret_cast<const __nv_bfloat162*>(&s_lo);
    const __nv_bfloat162* shi = reinterpret_cast<const __nv_bfloat162*>(&s_hi);
    float lo[4], hi[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float2 xx = __bfloat1622float2(xp[p]);  // x[2k], x[2k+1] with k = 4c + p
      const float2 cl = __bfloat1622float2(clo[p >> 1]);
      const float2 ch = __bfloat1622float2(chi[p >> 1]);
      const float2 sl = __bfloat1622float2(slo[p >> 1]);
      const float2 sh = __bfloat1622float2(shi[p >> 1]);
      const float ckl = (p & 1) ? cl.y : cl.x, ckh = (p & 1) ? ch.y : ch.x;
      const float skl = (p & 1) ? sl.y : sl.x, skh = (p & 1) ? sh.y : sh.x;
      lo[p] = xx.x * ckl - xx.y * skl;
      hi[p] = xx.y * ckh + xx.x * skh;
    }
    uint2 olo, ohi;
    const __nv_bfloat162 a0 = __floats2bfloat162_rn(lo[0], lo[1]);
    const __nv_bfloat162 a1 = __floats2bfloat162_rn(lo[2], lo[3]);
    const __nv_bfloat162 b0 = __floats2bfloat162_rn(hi[0], hi[1]);
    const __nv_bfloat162 b1 = __floats2bfloat162_rn(hi[2], hi[3]);
    olo.x = *reinterpret_cast<const uint32_t*>(&a0);
    olo.y = *reinterpret_cast<const uint32_t*>(&a1);
    ohi.x = *reinterpret_cast<const uint32_t*>(&b0);
    ohi.y = *reinterpret_cast<const uint32_t*>(&b1);
    __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>((is_q ? qo : ko) + lrow * D8);
    *reinterpret_cast<uint2*>(orow + 4 * c) = olo;
    *reinterpret_cast<uint2*>(orow + half + 4 * c) = ohi;
  }
}

// rope_dim % 16 == 0: one thread per (batch, position, 16-element chunk, group of 4 rows)
// where the rows of a (batch, position) are the q heads and then k.  The chunk's 8 rotation
// pairs k = 8c..8c+7 need cos/sin[k] and cos/sin[half + k] (one 16-byte load each), loaded
// once per thread for 4 rows instead of once per row; the 4 rows' loads are issued together.
constexpr int kRopeRows = 4;
__global__ void __launch_bounds__(256, 3)
    rope_heads_kernel(const uint4* __restrict__ q, const uint4* __restrict__ k,
                      const uint4* __restrict__ cos_t, const uint4* __restrict__ sin_t,
                      uint4* __restrict__ qo, uint4* __restrict__ ko, int64_t bs_rows,
                      int heads, int seq, int D) {
  const int D8 = D >> 3, D16 = D >> 4, H8 = D >> 4;  // H8: uint4 offset of the second half
  const int groups = (heads + 1 + kRopeRows - 1) / kRopeRows;
  const int64_t total = bs_rows * D16 * groups;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    // consecutive threads: chunks of one row, then positions (contiguous rows), then groups
    const int c = static_cast<int>(i % D16);
    const int64_t t = i / D16;
    const int64_t bs = t % bs_rows;  // b * seq + s
    const int g = static_cast<int>(t / bs_rows);
    const int64_t b = bs / seq, sp = bs - b * seq;
    // the chunk's cos/sin stay packed (16 registers) and are widened per row
    const uint4 cl4 = __ldg(cos_t + bs * D8 + c), ch4 = __ldg(cos_t + bs * D8 + H8 + c);
    const uint4 sl4 = __ldg(sin_t + bs * D8 + c), sh4 = __ldg(sin_t + bs * D8 + H8 + c);
    uint4 xv[kRopeRows][2];
    int64_t rows[kRopeRows];
#pragma unroll
    for (int j = 0; j < kRopeRows; ++j) {
      const int h = g * kRopeRows + j;  // h == heads: the k row
      rows[j] = h < heads ? (b * heads + h) * seq + sp : (h == heads ? bs : -1);
      if (rows[j] >= 0) {
        const uint4* src = (h < heads ? q : k) + rows[j] * D8 + 2 * c;
        xv[j][0] = __ldg(src);
        xv[j][1] = __ldg(src + 1);
      }
    }
#pragma unroll
    for (int j = 0; j < kRopeRows; ++j) {
      if (rows[j] < 0) continue;
      float x0[8], x1[8], cl[8], ch[8], sl[8], sh[8];
      bf16x8_to_f32(xv[j][0], x0);
      bf16x8_to_f32(xv[j][1], x1);
      bf16x8_to_f32(cl4, cl);
      bf16x8_to_f32(ch4, ch);
      bf16x8_to_f32(sl4, sl);
      bf16x8_to_f32(sh4, sh);
      float lo[8], hi[8];
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        const float xe = p < 4 ? x0[2 * p] : x1[2 * p - 8];
        const float xo = p < 4 ? x0[2 * p + 1] : x1[2 * p - 7];
        lo[p] = xe * cl[p] - xo * sl[p];
        hi[p] = xo * ch[p] + xe * sh[p];
      }
      uint4* dst = (g * kRopeRows + j < heads ? qo : ko) + rows[j] * D8;
      dst[c] = f32x8_to_bf16(lo);
      dst[H8 + c] = f32x8_to_bf16(hi);
    }
  }
}

// Scalar fallback for rope_dim not divisible by 8: one thread per rotation pair.
__global__ void rope_pair_kernel(const __nv_bfloat16* __restrict__ q,
                                 const __nv_bfloat16* __restrict__ k,
                                 const __nv_bfloat16* __restrict__ cos_t,
                                 const __nv_bfloat16* __restrict__ sin_t,
                                 __nv_bfloat16* __restrict__ qo, __nv_bfloat16* __restrict__ ko,
                                 int64_t q_rows, int64_t k_rows, int heads, int seq, int D) {
  const int half = D >> 1;
  const int64_t total = (q_rows + k_rows) * half;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / half;
    const int kk = static_cast<int>(i - row * half);
    const bool is_q = row < q_rows;
    const int64_t lrow = is_q ? row : row - q_rows;
    const int64_t cs_row =
        is_q ? (lrow / (static_cast<int64_t>(seq) * heads)) * seq + lrow % seq : lrow;
    const __nv_bfloat16* x = (is_q ? q : k) + lrow * D;
    const float x0 = __bfloat162float(x[2 * kk]), x1 = __bfloat162float(x[2 * kk + 1]);
    const __nv_bfloat16* cr = cos_t + cs_row * D;
    const __nv_bfloat16* sr = sin_t + cs_row * D;
    __nv_bfloat16* o = (is_q ? qo : ko) + lrow * D;
    o[kk] = __float2bfloat16_rn(x0 * __bfloat162float(cr[kk]) - x1 * __bfloat162float(sr[kk]));
    o[kk + half] = __float2bfloat16_rn(x1 * __bfloat162float(cr[kk + half]) +
                                       x0 * __bfloat162float(sr[kk + half]));
  }
}

// Opt a kernel into `bytes` of dynamic shared memory once per device (above 48 KB).
int smem_opt_in(const void* fn, int slot, int bytes, int device) {
  static std::mutex mu;
  static int done[1][64] = {};
  if (device < 0 || device >= 64) return fail(DS_ERR_UNSUPPORTED, "device ordinal %d", device);
  std::lock_guard<std::mutex> lock(mu);
  if (done[slot][device] < bytes) {
    DS_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done[slot][device] = bytes;
  }
  return DS_OK;
}

int grid_cap(int64_t items, int per_block, int num_sms) {
  const int64_t need = (items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(num_sms) * 8;
  return static_cast<int>(need < cap ? (need > 0 ? need : 1) : cap);
}

}  // namespace
}  // namespace ds

extern "C" {

int ds_rms_norm_strided(const void* input_bf16, int64_t in_stride, const float* weight,
                        void* output_bf16, int64_t out_stride, int rows, int hidden_size,
                        float eps, void* stream) {
  DS_REQUIRE(hidden_size > 0 && hidden_size % 2 == 0,
             "rms_norm: hidden_size must be even for bfloat162 vectorisation.");
  DS_REQUIRE(rows >= 0, "rms_norm: rows must be >= 0");
  DS_REQUIRE(in_stride >= hidden_size && out_stride >= hidden_size,
             "rms_norm: row strides must be >= hidden_size");
  if (rows == 0) return DS_OK;
  DS_REQUIRE(input_bf16 && weight && output_bf16, "rms_norm: null pointer");
  ds::DeviceInfo di;
  DS_TRY(ds::device_info(&di));
  const int vec_ok = (hidden_size % 8 == 0 && in_stride % 8 == 0 && out_stride % 8 == 0 &&
                      ds::aligned16(input_bf16) && ds::aligned16(output_bf16) &&
                      ds::aligned16(weight))
                         ? 1
                         : 0;
  if (vec_ok && hidden_size <= 512 && in_stride == hidden_size && out_stride == hidden_size) {
    int* status = ds::device_status_ptr();
    if (status == nullptr) return ds::fail(DS_ERR_CUDA, "device status word unavailable");
    const int ntiles = (rows + ds::kNormTileRows - 1) / ds::kNormTileRows;
    const int grid = ntiles < 2 * di.num_sms ? ntiles : 2 * di.num_sms;
    const int smem = ds::kNormStages * ds::kNormTileRows * hidden_size * 2;
    DS_TRY(ds::smem_opt_in(reinterpret_cast<const void*>(ds::rms_norm_ring_kernel), 0, smem,
                           di.device));
    ds::rms_norm_ring_kernel<<<grid, 256, smem, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(input_bf16), reinterpret_cast<const float4*>(weight),
        static_cast<uint4*>(output_bf16), rows, hidden_size, eps, status,
        2000LL * di.clock_khz);
    DS_LAUNCH_CHECK("rms_norm_ring_kernel");
    return DS_OK;
  }
  if (vec_ok && hidden_size <= 512) {
    const int grid = ds::grid_cap((static_cast<int64_t>(rows) + 1) / 2, 8, di.num_sms);
    ds::rms_norm_pair_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(input_bf16), in_stride / 8, reinterpret_cast<const float4*>(weight),
        static_cast<uint4*>(output_bf16), out_stride / 8, rows, hidden_size, eps);
    DS_LAUNCH_CHECK("rms_norm_pair_kernel");
    return DS_OK;
  }
  const int grid = ds::grid_cap(rows, 8, di.num_sms);
  ds::rms_norm_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(input_bf16), in_stride, weight,
      static_cast<__nv_bfloat16*>(output_bf16), out_stride, rows, hidden_size, eps, vec_ok);
  DS_LAUNCH_CHECK("rms_norm_kernel");
  return DS_OK;
}

int ds_rms_norm_residual(const void* input_bf16, const void* residual_bf16, const float* weight,
                         void* sum_out_bf16, void* normed_out_bf16, int rows, int hidden_size,
                         float eps, void* stream) {
  DS_REQUIRE(rows >= 0, "rms_norm_residual: rows must be >= 0");
  DS_REQUIRE(hidden_size > 0 && hidden_size % 8 == 0 && hidden_size <= 2048,
             "rms_norm_residual: hidden_size must be a multiple of 8, at most 2048");
  if (rows == 0) return DS_OK;
  DS_REQUIRE(input_bf16 && residual_bf16 && weight && sum_out_bf16 && normed_out_bf16,
             "rms_norm_residual: null pointer");
  DS_REQUIRE(ds::aligned16(input_bf16) && ds::aligned16(residual_bf16) && ds::aligned16(weight) &&
                 ds::aligned16(sum_out_bf16) && ds::aligned16(normed_out_bf16),
             "rms_norm_residual: pointers must be 16-byte aligned");
  ds::DeviceInfo di;
  DS_TRY(ds::device_info(&di));
  const int grid = ds::grid_cap(rows, 8, di.num_sms);
  ds::rms_norm_residual_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(input_bf16), static_cast<const uint4*>(residual_bf16),
      reinterpret_cast<const float4*>(weight), static_cast<uint4*>(sum_out_bf16),
      static_cast<uint4*>(normed_out_bf16), rows, hidden_size, eps);
  DS_LAUNCH_CHECK("rms_norm_residual_kernel");
  return DS_OK;
}

int ds_rms_norm(const void* input_bf16, const float* weight, void* output_bf16, int rows,
                int hidden_size, float eps, void* stream) {
  return ds_rms_norm_strided(input_bf16, hidden_size, weight, output_bf16, hidden_size, rows,
                             hidden_size, eps, stream);
}

int ds_rope(const void* q_pe_bf16, const void* k_pe_bf16, const void* cos_bf16,
            const void* sin_bf16, void* q_out_bf16, void* k_out_bf16, int bsz, int heads,
            int seq, int rope_dim, void* stream) {
  DS_REQUIRE(rope_dim > 0 && rope_dim % 2 == 0, "rope: rope_dim must be even.");
  DS_REQUIRE(bsz >= 0 && heads >= 1 && seq >= 0, "rope: bad shape");
  const int64_t q_rows = static_cast<int64_t>(bsz) * heads * seq;
  const int64_t k_rows = static_cast<int64_t>(bsz) * seq;
  if (q_rows + k_rows == 0) return DS_OK;
  DS_REQUIRE(q_pe_bf16 && k_pe_bf16 && cos_bf16 && sin_bf16 && q_out_bf16 && k_out_bf16,
             "rope: null pointer");
  ds::DeviceInfo di;
  DS_TRY(ds::device_info(&di));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = rope_dim % 8 == 0 && ds::aligned16(q_pe_bf16) && ds::aligned16(k_pe_bf16) &&
                   ds::aligned16(q_out_bf16) && ds::aligned16(k_out_bf16) &&
                   (reinterpret_cast<uintptr_t>(cos_bf16) & 7u) == 0 &&
                   (reinterpret_cast<uintptr_t>(sin_bf16) & 7u) == 0;
  const bool heads16 = vec && rope_dim % 16 == 0 && ds::aligned16(cos_bf16) && ds::aligned16(sin_bf16);
  if (heads16) {
    const int64_t bs_rows = static_cast<int64_t>(bsz) * seq;
    const int groups = (heads + 1 + ds::kRopeRows - 1) / ds::kRopeRows;
    const int grid = ds::grid_cap(bs_rows * (rope_dim / 16) * groups, 256, di.num_sms);
    ds::rope_heads_kernel<<<grid, 256, 0, s>>>(
        static_cast<const uint4*>(q_pe_bf16), static_cast<const uint4*>(k_pe_bf16),
        static_cast<const uint4*>(cos_bf16), static_cast<const uint4*>(sin_bf16),
        static_cast<uint4*>(q_out_bf16), static_cast<uint4*>(k_out_bf16), bs_rows, heads, seq,
        rope_dim);
  } else if (vec) {
    const int grid = ds::grid_cap((q_rows + k_rows) * (rope_dim / 8), 256, di.num_sms);
    ds::rope_vec_kernel<<<grid, 256, 0, s>>>(
        static_cast<const uint4*>(q_pe_bf16), static_cast<const uint4*>(k_pe_bf16),
        static_cast<const __nv_bfloat16*>(cos_bf16), static_cast<const __nv_bfloat16*>(sin_bf16),
        static_cast<uint4*>(q_out_bf16), static_cast<uint4*>(k_out_bf16), q_rows, k_rows, heads,
        seq, rope_dim);
  } else {
    const int grid = ds::grid_cap((q_rows + k_rows) * (rope_dim / 2), 256, di.num_sms);
    ds::rope_pair_kernel<<<grid, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(q_pe_bf16), static_cast<const __nv_bfloat16*>(k_pe_bf16),
        static_cast<const __nv_bfloat16*>(cos_bf16), static_cast<const __nv_bfloat16*>(sin_bf16),
        static_cast<__nv_bfloat16*>(q_out_bf16), static_cast<__nv_bfloat16*>(k_out_bf16), q_rows,
        k_rows, heads, seq, rope_dim);
  }
  DS_LAUNCH_CHECK("rope_kernel");
  return DS_OK;
}

}  // extern "C"

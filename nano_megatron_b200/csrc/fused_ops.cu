// Memory-bound fused kernels for sm_100a: RMSNorm fwd/bwd, SwiGLU backward,
// standalone RoPE, vocab-parallel embedding fwd/bwd, vocab-parallel
// cross-entropy (statistics + finish, or fused single pass for one shard),
// multi-tensor AdamW over flat fp32 buffers, and a grad-norm reduction.
//
// All kernels are vectorised to 16-byte accesses and sized as grid-stride
// loops over a multiple of the SM count, so they run at HBM3e bandwidth.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace nmb {
namespace fused {

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  f[0] = bf16_lo(v.x);
  f[1] = bf16_hi(v.x);
  f[2] = bf16_lo(v.y);
  f[3] = bf16_hi(v.y);
  f[4] = bf16_lo(v.z);
  f[5] = bf16_hi(v.z);
  f[6] = bf16_lo(v.w);
  f[7] = bf16_hi(v.w);
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 v;
  v.x = pack_bf16x2(f[0], f[1]);
  v.y = pack_bf16x2(f[2], f[3]);
  v.z = pack_bf16x2(f[4], f[5]);
  v.w = pack_bf16x2(f[6], f[7]);
  return v;
}
__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// ------------------------------------------------------------------ RMSNorm
// One warp per row; H = NCH * 256 so each lane owns NCH 16-byte chunks.
// y = bf16(bf16(x * rstd) * w), matching "normalise in fp32, cast, scale".
template <int NCH>
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                   const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y,
                                   int64_t ldy, float* __restrict__ rstd_out, int rows, float eps) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x / 32;
  constexpr int H = NCH * 256;
  for (int row = blockIdx.x * warps + threadIdx.x / 32; row < rows; row += gridDim.x * warps) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * ldx);
    float v[NCH][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      unpack8(xr[c * 32 + lane], v[c]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[c][e] * v[c][e];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / static_cast<float>(H) + eps);
    uint4* yr = reinterpret_cast<uint4*>(y + static_cast<int64_t>(row) * ldy);
    const uint4* wr = reinterpret_cast<const uint4*>(w);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      float wf[8], o[8];
      unpack8(wr[c * 32 + lane], wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = round_bf16(v[c][e] * r) * wf[e];
      yr[c * 32 + lane] = pack8(o);
    }
    if (lane == 0 && rstd_out != nullptr) rstd_out[row] = r;
  }
}

// dx = rstd * (w*dy - xhat * mean(xhat * w*dy)); dw += sum_rows dy * bf16(xhat).
// dw accumulates into an fp32 buffer (block-reduced in shared memory first).
template <int NCH>
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                   const __nv_bfloat16* __restrict__ w,
                                   const __nv_bfloat16* __restrict__ dy, int64_t lddy,
                                   const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx,
                                   int64_t lddx, float* __restrict__ dw,
                                   const __nv_bfloat16* __restrict__ dres, int64_t lddres,
                                   int rows) {
  constexpr int H = NCH * 256;
  __shared__ float sdw[H];
  for (int i = threadIdx.x; i < H; i += blockDim.x) sdw[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x / 32;
  // Narrow rows keep the weight in registers; wide rows re-read it (L1) to save registers.
  constexpr int WREG = NCH <= 4 ? NCH : 1;
  float wf[WREG][8];
  float dwacc[WREG][8];  // wide rows accumulate the weight gradient in shared memory
  const uint4* wr = reinterpret_cast<const uint4*>(w);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    if constexpr (NCH <= 4) {
      unpack8(wr[c * 32 + lane], wf[c]);
#pragma unroll
      for (int e = 0; e < 8; ++e) dwacc[c][e] = 0.f;
    }
  }
  for (int row = blockIdx.x * warps + threadIdx.x / 32; row < rows; row += gridDim.x * warps) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * ldx);
    const uint4* gr = reinterpret_cast<const uint4*>(dy + static_cast<int64_t>(row) * lddy);
    const float r = rstd[row];
    uint4* dr = reinterpret_cast<uint4*>(dx + static_cast<int64_t>(row) * lddx);
    const uint4* rr =
        dres != nullptr ? reinterpret_cast<const uint4*>(dres + static_cast<int64_t>(row) * lddres)
                        : nullptr;
    if constexpr (NCH <= 4) {
      // Narrow rows: keep x_hat and w*dy of the row in registers between the two sweeps.
      float xh[NCH][8], wg[NCH][8];
      float dot = 0.f;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        float xv[8], gv[8];
        unpack8(xr[c * 32 + lane], xv);
        unpack8(gr[c * 32 + lane], gv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          xh[c][e] = xv[e] * r;
          wg[c][e] = wf[c][e] * gv[e];
          dot += xh[c][e] * wg[c][e];
          dwacc[c][e] += gv[e] * round_bf16(xh[c][e]);
        }
      }
      dot = warp_sum(dot) / static_cast<float>(H);
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = r * (wg[c][e] - xh[c][e] * dot);
        if (rr != nullptr) {
          float rv[8];
          unpack8(rr[c * 32 + lane], rv);
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] += rv[e];
        }
        dr[c * 32 + lane] = pack8(o);
      }
    } else {
      // Wide rows (H >= 2048): two sweeps re-reading x and dy (L1-resident) so only the
      // weight-gradient accumulators stay live across the row.
      float dot = 0.f;
#pragma unroll 4
      for (int c = 0; c < NCH; ++c) {
        float xv[8], gv[8], wv[8];
        unpack8(xr[c * 32 + lane], xv);
        unpack8(gr[c * 32 + lane], gv);
        unpack8(wr[c * 32 + lane], wv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float xhv = xv[e] * r;
          dot += xhv * (wv[e] * gv[e]);
          if (dw != nullptr) atomicAdd(&sdw[(c * 32 + lane) * 8 + e], gv[e] * round_bf16(xhv));
        }
      }
      dot = warp_sum(dot) / static_cast<float>(H);
#pragma unroll 4
      for (int c = 0; c < NCH; ++c) {
        float xv[8], gv[8], wv[8], o[8];
        unpack8(xr[c * 32 + lane], xv);
        unpack8(gr[c * 32 + lane], gv);
        unpack8(wr[c * 32 + lane], wv);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = r * (wv[e] * gv[e] - xv[e] * r * dot);
        if (rr != nullptr) {
          float rv[8];
          unpack8(rr[c * 32 + lane], rv);
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] += rv[e];
        }
        dr[c * 32 + lane] = pack8(o);
      }
    }
  }
  if (dw != nullptr) {
    if constexpr (NCH <= 4) {
#pragma unroll
      for (int c = 0; c < NCH; ++c)
#pragma unroll
        for (int e = 0; e < 8; ++e) atomicAdd(&sdw[(c * 32 + lane) * 8 + e], dwacc[c][e]);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < H; i += blockDim.x) atomicAdd(&dw[i], sdw[i]);
  }
}

// ------------------------------------------------------------------ SwiGLU
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + __expf(-x)); }

// gu = [g | u] ([T, 2F]); h = silu(g) * u
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, int64_t ldgu,
                                  __nv_bfloat16* __restrict__ h, int64_t ldh, int T, int F) {
  const int64_t vec_per_row = F / 8;
  const int64_t total = static_cast<int64_t>(T) * vec_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vec_per_row, c = (i % vec_per_row) * 8;
    float g[8], u[8], o[8];
    unpack8(*reinterpret_cast<const uint4*>(gu + r * ldgu + c), g);
    unpack8(*reinterpret_cast<const uint4*>(gu + r * ldgu + F + c), u);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = g[e] * sigmoid_f(g[e]) * u[e];
    *reinterpret_cast<uint4*>(h + r * ldh + c) = pack8(o);
  }
}

// dgu = [dh * u * silu'(g) | dh * silu(g)]; may alias gu (in place).
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* gu, int64_t ldgu,
                                  const __nv_bfloat16* __restrict__ dh, int64_t lddh,
                                  __nv_bfloat16* dgu, int64_t lddgu, int T, int F) {
  const int64_t vec_per_row = F / 8;
  const int64_t total = static_cast<int64_t>(T) * vec_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vec_per_row, c = (i % vec_per_row) * 8;
    float g[8], u[8], d[8], dg[8], du[8];
    unpack8(*reinterpret_cast<const uint4*>(gu + r * ldgu + c), g);
    unpack8(*reinterpret_cast<const uint4*>(gu + r * ldgu + F + c), u);
    unpack8(*reinterpret_cast<const uint4*>(dh + r * lddh + c), d);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float s = sigmoid_f(g[e]);
      const float silu = g[e] * s;
      du[e] = d[e] * silu;
      dg[e] = d[e] * u[e] * s * (1.f + g[e] * (1.f - s));
    }
    *reinterpret_cast<uint4*>(dgu + r * lddgu + c) = pack8(dg);
    *reinterpret_cast<uint4*>(dgu + r * lddgu + F + c) = pack8(du);
  }
}

// ------------------------------------------------------------------ RoPE
// In-place rotate-half rotary embedding on the first `ncols` columns of each
// row of x ([rows, ld]); heads of size D; position of row r = pos[r % seq].
// sign = +1 applies the rotation, -1 its inverse (backward).
__global__ void rope_kernel(__nv_bfloat16* x, int64_t ld, int rows, int ncols, int D,
                            const int* __restrict__ pos, int seq, const float* __restrict__ inv_freq,
                            float sign) {
  const int half = D / 2;
  const int pairs_per_row = ncols / 2;
  const int64_t total = static_cast<int64_t>(rows) * pairs_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / pairs_per_row;
    const int pr = static_cast<int>(i % pairs_per_row);
    const int head = pr / half, c = pr % half;
    __nv_bfloat16* base = x + r * ld + head * D;
    const float ang = static_cast<float>(pos[r % seq]) * inv_freq[c];
    float sn, cs;
    sincosf(ang, &sn, &cs);
    sn *= sign;
    const float x1 = __bfloat162float(base[c]), x2 = __bfloat162float(base[c + half]);
    base[c] = __float2bfloat16_rn(x1 * cs - x2 * sn);
    base[c + half] = __float2bfloat16_rn(x2 * cs + x1 * sn);
  }
}

// ------------------------------------------------------------------ embedding
// out[t] = (vstart <= id < vstart + V) ? W[id - vstart] : 0, one warp per token.
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids,
                                     const __nv_bfloat16* __restrict__ w, int64_t V, int64_t vstart,
                                     __nv_bfloat16* __restrict__ out, int T, int H) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x / 32;
  const int nvec = H / 8;
  for (int t = blockIdx.x * warps + threadIdx.x / 32; t < T; t += gridDim.x * warps) {
    const int64_t id = ids[t] - vstart;
    const bool ok = id >= 0 && id < V;
    uint4* o = reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * H);
    const uint4* src = reinterpret_cast<const uint4*>(w + (ok ? id : 0) * H);
    for (int c = lane; c < nvec; c += 32) o[c] = ok ? src[c] : make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

// grad[id - vstart] += dy[t] (fp32 accumulation buffer).
__global__ void embedding_bwd_kernel(const int64_t* __restrict__ ids,
                                     const __nv_bfloat16* __restrict__ dy, int64_t lddy,
                                     float* __restrict__ grad, int64_t V, int64_t vstart, int T,
                                     int H) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x / 32;
  const int nvec = H / 8;
  for (int t = blockIdx.x * warps + threadIdx.x / 32; t < T; t += gridDim.x * warps) {
    const int64_t id = ids[t] - vstart;
    if (id < 0 || id >= V) continue;
    const uint4* g = reinterpret_cast<const uint4*>(dy + static_cast<int64_t>(t) * lddy);
    float* dst = grad + id * H;
    for (int c = lane; c < nvec; c += 32) {
      float f[8];
      unpack8(g[c], f);
      red_add_v4(dst + c * 8, f[0], f[1], f[2], f[3]);
      red_add_v4(dst + c * 8 + 4, f[4], f[5], f[6], f[7]);
    }
  }
}

// ------------------------------------------------------------------ deterministic mode
// Kernels used instead of the atomic reductions above while deterministic_mode() is on.
struct StridedRows {
  const __nv_bfloat16* base;
  int64_t ld;
  __device__ __forceinline__ uint4 operator()(int64_t t, int c) const {
    return reinterpret_cast<const uint4*>(base + t * ld)[c];
  }
};

// grad[id - vstart] += dy[t], tokens grouped by id and added in token order.
__global__ void embedding_bwd_sorted_kernel(const int64_t* __restrict__ sorted_ids,
                                            const int64_t* __restrict__ order,
                                            const __nv_bfloat16* __restrict__ dy, int64_t lddy,
                                            float* __restrict__ grad, int64_t V, int64_t vstart,
                                            int T, int H) {
  add_sorted_runs(sorted_ids, order, T, vstart, V, H, grad, StridedRows{dy, lddy});
}

// RMSNorm weight gradient, first pass: partial[chunk][c] = sum over the chunk's rows, in
// row order, of dy[r][c] * bf16(x[r][c] * rstd[r]) (the product the fused backward
// accumulates). One thread per column; slots_sum_kernel adds the chunks in order.
__global__ void rmsnorm_dw_partial_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                          const __nv_bfloat16* __restrict__ dy, int64_t lddy,
                                          const float* __restrict__ rstd, int rows, int H,
                                          int rows_per_chunk, float* __restrict__ partial) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  const int r0 = blockIdx.y * rows_per_chunk;
  const int r1 = min(rows, r0 + rows_per_chunk);
  float acc = 0.f;
  for (int r = r0; r < r1; ++r) {
    const float xh = __bfloat162float(x[static_cast<int64_t>(r) * ldx + c]) * rstd[r];
    acc += __bfloat162float(dy[static_cast<int64_t>(r) * lddy + c]) * round_bf16(xh);
  }
  partial[static_cast<int64_t>(blockIdx.y) * H + c] = acc;
}

// out[i] = (accumulate ? out[i] : 0) + slots[0][i] + slots[1][i] + ... + slots[S-1][i],
// summed in slot order. `vec`: n % 4 == 0 and both buffers 16-byte aligned.
__global__ void slots_sum_kernel(const float* __restrict__ slots, int S, int64_t n,
                                 float* __restrict__ out, int accumulate, int vec) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (vec) {
    const int64_t n4 = n / 4;
    for (int64_t i = first; i < n4; i += stride) {
      float4 a = accumulate ? reinterpret_cast<const float4*>(out)[i] : make_float4(0, 0, 0, 0);
      for (int sl = 0; sl < S; ++sl) {
        const float4 v = reinterpret_cast<const float4*>(slots + sl * n)[i];
        a.x += v.x;
        a.y += v.y;
        a.z += v.z;
        a.w += v.w;
      }
      reinterpret_cast<float4*>(out)[i] = a;
    }
  } else {
    for (int64_t i = first; i < n; i += stride) {
      float a = accumulate ? out[i] : 0.f;
      for (int sl = 0; sl < S; ++sl) a += slots[sl * n + i];
      out[i] = a;
    }
  }
}

// ------------------------------------------------------------------ cross-entropy
constexpr float kLog2eF = 1.4426950408889634f;
constexpr float kLn2F = 0.6931471805599453f;

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Block-wide (max, sum exp) of a bf16 row segment. Returns (max, sumexp rel. to max).
template <int NT>
__device__ __forceinline__ void row_max_sumexp(const __nv_bfloat16* row, int V, float& m_out,
                                               float& s_out) {
  __shared__ float red_m[NT / 32], red_s[NT / 32];
  float m = -INFINITY, s = 0.f;
  const int nvec = V / 8;
  for (int c = threadIdx.x; c < nvec; c += NT) {
    float f[8];
    unpack8(reinterpret_cast<const uint4*>(row)[c], f);
    float lm = f[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) lm = fmaxf(lm, f[e]);
    const float nm = fmaxf(m, lm);
    s = s * ex2f((m - nm) * kLog2eF);
#pragma unroll
    for (int e = 0; e < 8; ++e) s += ex2f((f[e] - nm) * kLog2eF);
    m = nm;
  }
  // warp reduce (m, s)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * ex2f((m - nm) * kLog2eF)) +
        (om == -INFINITY ? 0.f : os * ex2f((om - nm) * kLog2eF));
    m = nm;
  }
  const int w = threadIdx.x / 32;
  if ((threadIdx.x & 31) == 0) {
    red_m[w] = m;
    red_s[w] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = red_m[0], Ssum = red_s[0];
    for (int i = 1; i < NT / 32; ++i) {
      const float nm = fmaxf(M, red_m[i]);
      Ssum = (M == -INFINITY ? 0.f : Ssum * ex2f((M - nm) * kLog2eF)) +
             (red_m[i] == -INFINITY ? 0.f : red_s[i] * ex2f((red_m[i] - nm) * kLog2eF));
      M = nm;
    }
    red_m[0] = M;
    red_s[0] = Ssum;
  }
  __syncthreads();
  m_out = red_m[0];
  s_out = red_s[0];
  __syncthreads();
}

// Per-row partial statistics of one vocabulary shard: (max, sumexp, target logit).
template <int NT>
__global__ void __launch_bounds__(NT) ce_stats_kernel(const __nv_bfloat16* __restrict__ logits,
                                                      int64_t ld, const int64_t* __restrict__ labels,
                                                      int64_t vstart, int V, int T,
                                                      float* __restrict__ stats) {
  const int t = blockIdx.x;
  if (t >= T) return;
  const __nv_bfloat16* row = logits + static_cast<int64_t>(t) * ld;
  float m, s;
  row_max_sumexp<NT>(row, V, m, s);
  if (threadIdx.x == 0) {
    const int64_t lab = labels[t];
    const int64_t li = lab - vstart;
    const float tgt = (lab >= 0 && li >= 0 && li < V) ? __bfloat162float(row[li]) : 0.f;
    stats[t * 3 + 0] = m;
    stats[t * 3 + 1] = s;
    stats[t * 3 + 2] = tgt;
  }
}

// Combine the statistics of `shards` vocabulary shards ([shards, T, 3]),
// write per-row loss (0 for ignored rows) and overwrite the local logits with
// d loss_row / d logits = softmax - onehot (0 for ignored rows).
template <int NT>
__global__ void __launch_bounds__(NT) ce_finish_kernel(__nv_bfloat16* logits, int64_t ld,
                                                       const int64_t* __restrict__ labels,
                                                       int64_t vstart, int V, int T,
                                                       const float* __restrict__ stats, int shards,
                                                       float* __restrict__ loss_row,
                                                       int write_grad) {
  const int t = blockIdx.x;
  if (t >= T) return;
  __shared__ float s_lse;
  const int64_t lab = labels[t];
  const bool valid = lab >= 0;
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int r = 0; r < shards; ++r) M = fmaxf(M, stats[(static_cast<int64_t>(r) * T + t) * 3]);
    float S = 0.f, tgt = 0.f;
    for (int r = 0; r < shards; ++r) {
      const float* st = stats + (static_cast<int64_t>(r) * T + t) * 3;
      if (st[0] != -INFINITY) S += st[1] * ex2f((st[0] - M) * kLog2eF);
      tgt += st[2];
    }
    const float lse = M + __log2f(S) * kLn2F;
    s_lse = lse;
    loss_row[t] = valid ? (lse - tgt) : 0.f;
  }
  __syncthreads();
  if (!write_grad) return;
  const float lse = s_lse;
  __nv_bfloat16* row = logits + static_cast<int64_t>(t) * ld;
  const int64_t li = lab - vstart;
  const int nvec = V / 8;
  for (int c = threadIdx.x; c < nvec; c += NT) {
    uint4* p = reinterpret_cast<uint4*>(row) + c;
    float f[8];
    unpack8(*p, f);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float gval = valid ? ex2f((f[e] - lse) * kLog2eF) : 0.f;
      if (valid && c * 8 + e == li) gval -= 1.f;
      f[e] = gval;
    }
    *p = pack8(f);
  }
}

// Single-shard fused version: statistics + finish in one pass per row.
template <int NT>
__global__ void __launch_bounds__(NT) ce_fused_kernel(__nv_bfloat16* logits, int64_t ld,
                                                      const int64_t* __restrict__ labels, int V,
                                                      int T, float* __restrict__ loss_row,
                                                      int write_grad) {
  const int t = blockIdx.x;
  if (t >= T) return;
  __nv_bfloat16* row = logits + static_cast<int64_t>(t) * ld;
  float m, s;
  row_max_sumexp<NT>(row, V, m, s);
  const int64_t lab = labels[t];
  const bool valid = lab >= 0;
  const float lse = m + __log2f(s) * kLn2F;
  if (threadIdx.x == 0) {
    const float tgt = (valid && lab < V) ? __bfloat162float(row[lab]) : 0.f;
    loss_row[t] = valid ? lse - tgt : 0.f;
  }
  __syncthreads();
  if (!write_grad) return;
  const int nvec = V / 8;
  for (int c = threadIdx.x; c < nvec; c += NT) {
    uint4* p = reinterpret_cast<uint4*>(row) + c;
    float f[8];
    unpack8(*p, f);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float gval = valid ? ex2f((f[e] - lse) * kLog2eF) : 0.f;
      if (valid && c * 8 + e == lab) gval -= 1.f;
      f[e] = gval;
    }
    *p = pack8(f);
  }
}

// (max, sum exp) of a row from `n` partial pairs written by the LM-head GEMM epilogue,
// merged by one warp.
__device__ __forceinline__ void merge_parts_warp(const float2* __restrict__ parts, int n,
                                                 float& m_out, float& s_out) {
  const int lane = threadIdx.x & 31;
  float m = -INFINITY, s = 0.f;
  for (int i = lane; i < n; i += 32) {
    const float2 q = parts[i];
    const float nm = fmaxf(m, q.x);
    if (nm != -INFINITY)
      s = (m == -INFINITY ? 0.f : s * ex2f((m - nm) * kLog2eF)) +
          (q.x == -INFINITY ? 0.f : q.y * ex2f((q.x - nm) * kLog2eF));
    m = nm;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    if (nm != -INFINITY)
      s = (m == -INFINITY ? 0.f : s * ex2f((m - nm) * kLog2eF)) +
          (om == -INFINITY ? 0.f : os * ex2f((om - nm) * kLog2eF));
    m = nm;
  }
  m_out = m;
  s_out = s;
}

// Cross-entropy over the whole vocabulary from the LM-head GEMM's per-tile statistics:
// row loss, and the logits overwritten by softmax - onehot. One pass over the logits (the
// statistics pass ran inside the GEMM).
template <int NT>
__global__ void __launch_bounds__(NT) ce_parts_finish_kernel(
    __nv_bfloat16* logits, int64_t ld, const int64_t* __restrict__ labels, int V, int T,
    const float2* __restrict__ parts, int nparts, float* __restrict__ loss_row, int write_grad) {
  const int t = blockIdx.x;
  if (t >= T) return;
  __shared__ float s_lse;
  __nv_bfloat16* row = logits + static_cast<int64_t>(t) * ld;
  const int64_t lab = labels[t];
  const bool valid = lab >= 0;
  if (threadIdx.x < 32) {
    float m, sx;
    merge_parts_warp(parts + static_cast<int64_t>(t) * nparts, nparts, m, sx);
    if (threadIdx.x == 0) {
      const float lse = m + __log2f(sx) * kLn2F;
      const float tgt = (valid && lab < V) ? __bfloat162float(row[lab]) : 0.f;
      loss_row[t] = valid ? lse - tgt : 0.f;
      s_lse = lse;
    }
  }
  __syncthreads();
  if (!write_grad) return;
  const float lse = s_lse;
  const int nvec = V / 8;
  for (int c = threadIdx.x; c < nvec; c += NT) {
    uint4* q = reinterpret_cast<uint4*>(row) + c;
    float f[8];
    unpack8(*q, f);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float gval = valid ? ex2f((f[e] - lse) * kLog2eF) : 0.f;
      if (valid && c * 8 + e == lab) gval -= 1.f;
      f[e] = gval;
    }
    *q = pack8(f);
  }
}

// ------------------------------------------------------------------ AdamW
// Decoupled-weight-decay Adam over flat fp32 buffers (torch.optim.AdamW
// semantics): p *= 1 - lr*wd; m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2;
// p -= (lr / bc1) * m / (sqrt(v) / sqrt(bc2) + eps). Gradients are scaled by
// *grad_scale (the clip coefficient, kept on device) when given. Optionally
// writes the bf16 copy of the updated parameter.
struct AdamHyper {
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt;
};

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g,
                             float* __restrict__ m, float* __restrict__ v,
                             __nv_bfloat16* __restrict__ p_bf16, int64_t n, AdamHyper hp,
                             const float* __restrict__ grad_scale,
                             const float* __restrict__ lr_ptr) {
  const float gs = grad_scale != nullptr ? *grad_scale : 1.f;
  const float lr = lr_ptr != nullptr ? *lr_ptr : hp.lr;
  const float step = lr / hp.bc1;
  const float decay = 1.f - lr * hp.wd;
  const int64_t n4 = n / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += stride) {
    float4 pv = reinterpret_cast<float4*>(p)[i];
    const float4 gv = reinterpret_cast<const float4*>(g)[i];
    float4 mv = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pp = &pv.x;
    const float* gp = &gv.x;
    float* mp = &mv.x;
    float* vp = &vv.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float gr = gp[e] * gs;
      pp[e] *= decay;
      mp[e] = hp.beta1 * mp[e] + (1.f - hp.beta1) * gr;
      vp[e] = hp.beta2 * vp[e] + (1.f - hp.beta2) * gr * gr;
      pp[e] -= step * mp[e] / (sqrtf(vp[e]) / hp.bc2_sqrt + hp.eps);
    }
    reinterpret_cast<float4*>(p)[i] = pv;
    reinterpret_cast<float4*>(m)[i] = mv;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (p_bf16 != nullptr) {
      uint2 o;
      o.x = pack_bf16x2(pv.x, pv.y);
      o.y = pack_bf16x2(pv.z, pv.w);
      reinterpret_cast<uint2*>(p_bf16)[i] = o;
    }
  }
  // scalar tail
  for (int64_t i = n4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += stride) {
    const float gr = g[i] * gs;
    float pe = p[i] * decay;
    m[i] = hp.beta1 * m[i] + (1.f - hp.beta1) * gr;
    v[i] = hp.beta2 * v[i] + (1.f - hp.beta2) * gr * gr;
    pe -= step * m[i] / (sqrtf(v[i]) / hp.bc2_sqrt + hp.eps);
    p[i] = pe;
    if (p_bf16 != nullptr) p_bf16[i] = __float2bfloat16_rn(pe);
  }
}

// Per-block partial sum of squares (fp32 input); partials[blockIdx.x].
__global__ void sumsq_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ partials) {
  float acc = 0.f;
  const int64_t n4 = n / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += stride) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (int64_t i = n4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += stride)
    acc += x[i] * x[i];
  acc = warp_sum(acc);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) partials[blockIdx.x] = v;
  }
}

// y = x * (*scale) (fp32, in place allowed) — used for DP averaging of flat grads.
__global__ void scale_kernel(float* __restrict__ x, int64_t n, float s) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride)
    x[i] *= s;
}

}  // namespace fused
}  // namespace nmb

using namespace nmb;
using namespace nmb::fused;

static int grid_for(int64_t work, int threads) {
  int dev;
  cudaGetDevice(&dev);
  int sms;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = (work + threads - 1) / threads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, sms * 8)));
}

#define NMB_CHECK_BF16(t) \
  TORCH_CHECK((t).is_cuda() && (t).scalar_type() == at::kBFloat16, #t " must be CUDA bf16")

namespace nmb {
namespace {
std::atomic<bool> g_deterministic{false};
}  // namespace
bool deterministic_mode() { return g_deterministic.load(std::memory_order_relaxed); }
}  // namespace nmb

void set_deterministic(bool on) { nmb::g_deterministic.store(on, std::memory_order_relaxed); }
bool get_deterministic() { return nmb::deterministic_mode(); }

// out (+)= sum over the leading dimension of `slots` ([S, out.numel()] fp32), in order.
void slots_sum(at::Tensor slots, at::Tensor out, bool accumulate) {
  TORCH_CHECK(slots.is_cuda() && slots.scalar_type() == at::kFloat && slots.is_contiguous());
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous());
  const int64_t n = out.numel();
  TORCH_CHECK(n > 0 && slots.numel() % n == 0, "slots_sum: slots must be [S, out.numel()]");
  const int64_t S = slots.numel() / n;
  TORCH_CHECK(S < (1ll << 31));
  const at::cuda::CUDAGuard guard(out.device());
  const bool vec = n % 4 == 0 && (reinterpret_cast<uintptr_t>(slots.data_ptr()) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15u) == 0;
  slots_sum_kernel<<<grid_for(vec ? n / 4 : n, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      slots.data_ptr<float>(), static_cast<int>(S), n, out.data_ptr<float>(),
      accumulate ? 1 : 0, vec ? 1 : 0); NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rmsnorm_fwd(at::Tensor x, at::Tensor w, at::Tensor y, at::Tensor rstd, double eps) {
  NMB_CHECK_BF16(x);
  NMB_CHECK_BF16(w);
  NMB_CHECK_BF16(y);
  const int64_t H = x.size(-1);
  TORCH_CHECK(H % 256 == 0 && H <= 8192, "rmsnorm: hidden size must be a multiple of 256");
  TORCH_CHECK(x.stride(-1) == 1 && y.stride(-1) == 1 && w.is_contiguous());
  const int rows = static_cast<int>(x.numel() / H);
  const int64_t ldx = x.dim() >= 2 ? x.stride(-2) : H;
  const int64_t ldy = y.dim() >= 2 ? y.stride(-2) : H;
  const at::cuda::CUDAGuard guard(x.device());
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  const int threads = 256;
  const int blocks = std::max(1, std::min((rows + 7) / 8, 148 * 16));
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  float* rp = rstd.data_ptr<float>();
  const float e = static_cast<float>(eps);
  switch (H / 256) {
    case 1: rmsnorm_fwd_kernel<1><<<blocks, threads, 0, s>>>(xp, ldx, wp, yp, ldy, rp, rows, e); NMB_LAUNCHED(1); break;
    case 2: rmsnorm_fwd_kernel<2><<<blocks, threads, 0, s>>>(xp, ldx, wp, yp, ldy, rp, rows, e); NMB_LAUNCHED(1); break;
    case 4: rmsnorm_fwd_kernel<4><<<blocks, threads, 0, s>>>(xp, ldx, wp, yp, ldy, rp, rows, e); NMB_LAUNCHED(1); break;
    case 8: rmsnorm_fwd_kernel<8><<<blocks, threads, 0, s>>>(xp, ldx, wp, yp, ldy, rp, rows, e); NMB_LAUNCHED(1); break;
    case 16: rmsnorm_fwd_kernel<16><<<blocks, threads, 0, s>>>(xp, ldx, wp, yp, ldy, rp, rows, e); NMB_LAUNCHED(1); break;
    default: TORCH_CHECK(false, "rmsnorm: unsupported hidden size ", H);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dx = RMSNorm backward (+ dres, the residual branch's gradient, when given).
void rmsnorm_bwd(at::Tensor x, at::Tensor w, at::Tensor dy, at::Tensor rstd, at::Tensor dx,
                 c10::optional<at::Tensor> dw, c10::optional<at::Tensor> dres) {
  NMB_CHECK_BF16(x);
  NMB_CHECK_BF16(dy);
  NMB_CHECK_BF16(dx);
  const int64_t H = x.size(-1);
  TORCH_CHECK(H % 256 == 0 && H <= 4096, "rmsnorm_bwd: hidden size must be 256..4096, /256");
  const int rows = static_cast<int>(x.numel() / H);
  const at::cuda::CUDAGuard guard(x.device());
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  const int threads = 256;
  const int blocks = std::max(1, std::min((rows + 7) / 8, 148 * 2));
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto gp = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  auto dxp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  float* dwp = nullptr;
  if (dw.has_value()) {
    TORCH_CHECK(dw->scalar_type() == at::kFloat && dw->is_contiguous());
    dwp = dw->data_ptr<float>();
  }
  const int64_t ldx = x.stride(-2), lddy = dy.stride(-2), lddx = dx.stride(-2);
  const float* rp = rstd.data_ptr<float>();
  const __nv_bfloat16* rsp = nullptr;
  int64_t ldr = 0;
  if (dres.has_value()) {
    NMB_CHECK_BF16(*dres);
    rsp = reinterpret_cast<const __nv_bfloat16*>(dres->data_ptr());
    ldr = dres->stride(-2);
  }
  // Deterministic mode: the fused kernel skips dw; two fixed-order passes add it.
  float* const dw_out = dwp;
  if (deterministic_mode()) dwp = nullptr;
  switch (H / 256) {
    case 1: rmsnorm_bwd_kernel<1><<<blocks, threads, 0, s>>>(xp, ldx, wp, gp, lddy, rp, dxp, lddx, dwp, rsp, ldr, rows); NMB_LAUNCHED(1); break;
    case 2: rmsnorm_bwd_kernel<2><<<blocks, threads, 0, s>>>(xp, ldx, wp, gp, lddy, rp, dxp, lddx, dwp, rsp, ldr, rows); NMB_LAUNCHED(1); break;
    case 4: rmsnorm_bwd_kernel<4><<<blocks, threads, 0, s>>>(xp, ldx, wp, gp, lddy, rp, dxp, lddx, dwp, rsp, ldr, rows); NMB_LAUNCHED(1); break;
    case 8: rmsnorm_bwd_kernel<8><<<blocks, threads, 0, s>>>(xp, ldx, wp, gp, lddy, rp, dxp, lddx, dwp, rsp, ldr, rows); NMB_LAUNCHED(1); break;
    case 16: rmsnorm_bwd_kernel<16><<<blocks, threads, 0, s>>>(xp, ldx, wp, gp, lddy, rp, dxp, lddx, dwp, rsp, ldr, rows); NMB_LAUNCHED(1); break;
    default: TORCH_CHECK(false, "rmsnorm_bwd: unsupported hidden size ", H);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (dw_out != nullptr && dwp == nullptr && rows > 0) {
    const int nchunks0 = std::min(rows, 4 * 148);
    const int per = (rows + nchunks0 - 1) / nchunks0;
    const int nchunks = (rows + per - 1) / per;
    at::Tensor partial = at::empty({nchunks, H}, x.options().dtype(at::kFloat));
    rmsnorm_dw_partial_kernel<<<dim3(static_cast<unsigned>((H + 255) / 256), nchunks), 256, 0,
                                s>>>(xp, ldx, gp, lddy, rp, rows, static_cast<int>(H), per,
                                     partial.data_ptr<float>()); NMB_LAUNCHED(1);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    slots_sum(partial, *dw, true);
  }
}

void swiglu_fwd(at::Tensor gu, at::Tensor h) {
  NMB_CHECK_BF16(gu);
  NMB_CHECK_BF16(h);
  const int T = gu.size(0), F = h.size(1);
  TORCH_CHECK(gu.size(1) == 2 * F && F % 8 == 0, "swiglu: bad shapes");
  const at::cuda::CUDAGuard guard(gu.device());
  const int64_t work = static_cast<int64_t>(T) * (F / 8);
  swiglu_fwd_kernel<<<grid_for(work, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), gu.stride(0),
      reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), h.stride(0), T, F); NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void swiglu_bwd(at::Tensor gu, at::Tensor dh, at::Tensor dgu) {
  NMB_CHECK_BF16(gu);
  NMB_CHECK_BF16(dh);
  NMB_CHECK_BF16(dgu);
  const int T = gu.size(0), F = dh.size(1);
  TORCH_CHECK(gu.size(1) == 2 * F && dgu.size(1) == 2 * F && F % 8 == 0, "swiglu_bwd: bad shapes");
  const at::cuda::CUDAGuard guard(gu.device());
  const int64_t work = static_cast<int64_t>(T) * (F / 8);
  swiglu_bwd_kernel<<<grid_for(work, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), gu.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(dh.data_ptr()), dh.stride(0),
      reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), dgu.stride(0), T, F); NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope_inplace(at::Tensor x, int64_t ncols, int64_t head_dim, at::Tensor pos, at::Tensor inv_freq,
                  bool inverse) {
  NMB_CHECK_BF16(x);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "rope: x must be 2-D row-major");
  TORCH_CHECK(ncols % head_dim == 0 && head_dim % 2 == 0);
  const int rows = x.size(0);
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t work = static_cast<int64_t>(rows) * (ncols / 2);
  rope_kernel<<<grid_for(work, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), x.stride(0), rows, ncols, head_dim,
      pos.data_ptr<int>(), pos.numel(), inv_freq.data_ptr<float>(), inverse ? -1.f : 1.f); NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding_fwd(at::Tensor ids, at::Tensor w, int64_t vstart, at::Tensor out) {
  NMB_CHECK_BF16(w);
  NMB_CHECK_BF16(out);
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous());
  const int T = ids.numel();
  const int H = w.size(1);
  TORCH_CHECK(H % 8 == 0 && w.is_contiguous() && out.is_contiguous());
  const at::cuda::CUDAGuard guard(w.device());
  const int blocks = std::max(1, std::min((T + 7) / 8, 148 * 16));
  embedding_fwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), w.size(0),
      vstart, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), T, H); NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding_bwd(at::Tensor ids, at::Tensor dy, at::Tensor grad, int64_t vstart) {
  NMB_CHECK_BF16(dy);
  TORCH_CHECK(grad.scalar_type() == at::kFloat && grad.is_contiguous());
  const int T = ids.numel();
  const int H = grad.size(1);
  TORCH_CHECK(H % 8 == 0);
  const at::cuda::CUDAGuard guard(dy.device());
  const int blocks = std::max(1, std::min((T + 7) / 8, 148 * 16));
  if (deterministic_mode()) {
    TORCH_CHECK(ids.scalar_type() == at::kLong && dy.stride(1) == 1 && dy.stride(0) % 8 == 0);
    if (T == 0) return;
    const auto sorted = at::sort(ids.reshape({-1}), /*stable=*/true, 0, false);
    const at::Tensor sid = std::get<0>(sorted).contiguous(), ord = std::get<1>(sorted).contiguous();
    embedding_bwd_sorted_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        sid.data_ptr<int64_t>(), ord.data_ptr<int64_t>(),
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), dy.stride(0),
        grad.data_ptr<float>(), grad.size(0), vstart, T, H); NMB_LAUNCHED(1);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  embedding_bwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
      dy.stride(0), grad.data_ptr<float>(), grad.size(0), vstart, T, H); NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_stats(at::Tensor logits, at::Tensor labels, int64_t vstart, at::Tensor stats) {
  NMB_CHECK_BF16(logits);
  const int T = logits.size(0), V = logits.size(1);
  TORCH_CHECK(V % 8 == 0 && logits.stride(1) == 1);
  const at::cuda::CUDAGuard guard(logits.device());
  ce_stats_kernel<256><<<T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
      labels.data_ptr<int64_t>(), vstart, V, T, stats.data_ptr<float>()); NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_finish(at::Tensor logits, at::Tensor labels, int64_t vstart, at::Tensor stats,
               int64_t shards, at::Tensor loss_row, bool write_grad) {
  NMB_CHECK_BF16(logits);
  const int T = logits.size(0), V = logits.size(1);
  const at::cuda::CUDAGuard guard(logits.device());
  ce_finish_kernel<256><<<T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
      labels.data_ptr<int64_t>(), vstart, V, T, stats.data_ptr<float>(), shards,
      loss_row.data_ptr<float>(), write_grad ? 1 : 0); NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_fused(at::Tensor logits, at::Tensor labels, at::Tensor loss_row, bool write_grad) {
  NMB_CHECK_BF16(logits);
  const int T = logits.size(0), V = logits.size(1);
  TORCH_CHECK(V % 8 == 0 && logits.stride(1) == 1);
  const at::cuda::CUDAGuard guard(logits.device());
  ce_fused_kernel<256><<<T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
      labels.data_ptr<int64_t>(), V, T, loss_row.data_ptr<float>(), write_grad ? 1 : 0); NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_from_parts(at::Tensor logits, at::Tensor labels, at::Tensor parts, int64_t nparts,
                   at::Tensor loss_row, bool write_grad) {
  NMB_CHECK_BF16(logits);
  const int T = logits.size(0), V = logits.size(1);
  TORCH_CHECK(V % 8 == 0 && logits.stride(1) == 1 && logits.stride(0) % 8 == 0);
  TORCH_CHECK(parts.is_cuda() && parts.scalar_type() == at::kFloat && parts.is_contiguous() &&
                  parts.numel() >= static_cast<int64_t>(T) * nparts * 2 && nparts >= 1,
              "ce_from_parts: parts must hold T x nparts (max, sum exp) pairs");
  TORCH_CHECK(labels.is_cuda() && labels.scalar_type() == at::kLong && labels.numel() == T);
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(logits.device());
  ce_parts_finish_kernel<256><<<T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
      labels.data_ptr<int64_t>(), V, T, reinterpret_cast<const float2*>(parts.data_ptr<float>()),
      static_cast<int>(nparts), loss_row.data_ptr<float>(), write_grad ? 1 : 0);
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v,
                c10::optional<at::Tensor> p_bf16, double lr, double beta1, double beta2,
                double eps, double wd, int64_t step, c10::optional<at::Tensor> grad_scale,
                c10::optional<at::Tensor> lr_t) {
  TORCH_CHECK(p.scalar_type() == at::kFloat && g.scalar_type() == at::kFloat &&
              m.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat);
  TORCH_CHECK(p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous());
  const int64_t n = p.numel();
  TORCH_CHECK(g.numel() == n && m.numel() == n && v.numel() == n);
  AdamHyper hp;
  hp.lr = static_cast<float>(lr);
  hp.beta1 = static_cast<float>(beta1);
  hp.beta2 = static_cast<float>(beta2);
  hp.eps = static_cast<float>(eps);
  hp.wd = static_cast<float>(wd);
  hp.bc1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  hp.bc2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  __nv_bfloat16* pb = nullptr;
  if (p_bf16.has_value()) {
    NMB_CHECK_BF16(*p_bf16);
    TORCH_CHECK(p_bf16->numel() == n && p_bf16->is_contiguous());
    pb = reinterpret_cast<__nv_bfloat16*>(p_bf16->data_ptr());
  }
  const at::cuda::CUDAGuard guard(p.device());
  adamw_kernel<<<grid_for(n / 4 + 1, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), pb, n,
      hp, grad_scale.has_value() ? grad_scale->data_ptr<float>() : nullptr,
      lr_t.has_value() ? lr_t->data_ptr<float>() : nullptr); NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

at::Tensor sumsq_partials(at::Tensor x) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous());
  const at::cuda::CUDAGuard guard(x.device());
  const int blocks = grid_for(x.numel() / 4 + 1, 256);
  auto out = at::empty({blocks}, x.options());
  sumsq_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(x.data_ptr<float>(),
                                                                    x.numel(), out.data_ptr<float>()); NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

void scale_inplace(at::Tensor x, double s) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous());
  const at::cuda::CUDAGuard guard(x.device());
  scale_kernel<<<grid_for(x.numel(), 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), x.numel(), static_cast<float>(s)); NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ dropout (Philox)
// Counter-based dropout: element i keeps with probability 1 - p according to
// Philox-4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as
// 1, 2, 3", SC 2011) keyed by a 64-bit seed, counter = i / 4, lane = i % 4. The mask is
// a pure function of (seed, i), so the backward pass regenerates it instead of storing
// it. y = x * keep / (1 - p).
namespace nmb {
namespace fused {

__device__ __forceinline__ uint4 philox4x32_10(uint4 ctr, uint2 key) {
  constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u;  // multipliers (paper, Table 2)
  constexpr uint32_t kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;  // key schedule (Weyl) constants
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(kM0, ctr.x), lo0 = kM0 * ctr.x;
    const uint32_t hi1 = __umulhi(kM1, ctr.z), lo1 = kM1 * ctr.z;
    ctr = make_uint4(hi1 ^ ctr.y ^ key.x, lo1, hi0 ^ ctr.w ^ key.y, lo0);
    key.x += kW0;
    key.y += kW1;
  }
  return ctr;
}

__global__ void dropout_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                               int64_t n, uint32_t keep_threshold, float scale, uint2 key) {
  const int64_t groups = (n + 3) / 4;
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < groups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 r = philox4x32_10(
        make_uint4(static_cast<uint32_t>(g), static_cast<uint32_t>(g >> 32), 0u, 0u), key);
    const uint32_t u[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t i = g * 4 + j;
      if (i < n) {
        const float v = __bfloat162float(x[i]);
        y[i] = __float2bfloat16_rn(u[j] < keep_threshold ? v * scale : 0.0f);
      }
    }
  }
}

}  // namespace fused
}  // namespace nmb

// y = dropout(x) with the mask of (seed, element index); call with dy/dx for the backward.
void dropout_apply(at::Tensor x, at::Tensor y, double p, int64_t seed) {
  NMB_CHECK_BF16(x);
  NMB_CHECK_BF16(y);
  TORCH_CHECK(x.is_contiguous() && y.is_contiguous() && x.numel() == y.numel());
  TORCH_CHECK(p >= 0.0 && p < 1.0, "dropout probability must be in [0, 1)");
  const int64_t n = x.numel();
  if (n == 0) return;
  const double keep = 1.0 - p;
  const uint32_t thr = keep >= 1.0 ? 0xFFFFFFFFu
                                   : static_cast<uint32_t>(keep * 4294967296.0);
  const uint64_t s = static_cast<uint64_t>(seed);
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t groups = (n + 3) / 4;
  nmb::fused::dropout_kernel<<<grid_for(groups, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), n, thr, static_cast<float>(1.0 / keep),
      make_uint2(static_cast<uint32_t>(s), static_cast<uint32_t>(s >> 32)));
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Causal flash attention, forward and backward, for sm_100a.
//
// Layout: q, k, v are read in place from the fused QKV projection output
// ([tokens, (Hq + 2 Hkv) * D] bf16, arbitrary row/batch strides), so no
// transpose or repeat_interleave is ever materialised; GQA is native (a KV
// head serves Hq / Hkv query heads). Causality is decided by absolute
// positions (q_offset + i vs k_offset + j) so the same kernels serve local
// attention and the context-parallel all-gather / ring variants; key blocks
// that lie entirely above the diagonal are skipped.
//
// Softmax runs in base 2: scores are pre-multiplied by softmax_scale*log2(e);
// the saved log-sum-exp `lse` is in the same base-2 units.
//
// Backward (one CTA per key block and KV head, looping over the query heads
// of its group): dK/dV accumulate in registers, dQ is accumulated in fp32
// with vector reductions and converted (plus inverse RoPE) by a small tail
// kernel. Inverse RoPE for dK is applied in registers before the store, so the
// QKV weight-gradient GEMM consumes pre-rotation gradients directly.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace nmb {
namespace attn {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const uint32_t s = smem_u32(smem);
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Swizzled [rows x D] bf16 tile: 16-byte chunk c of row r lives at chunk
// (c & ~7) | ((c ^ r) & 7). Returns a byte offset.
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int col) {
  const int chunk = col >> 3;
  const int phys = (chunk & ~7) | ((chunk ^ row) & 7);
  return static_cast<uint32_t>(row * D * 2 + phys * 16 + (col & 7) * 2);
}

struct FwdParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t q_row, k_row, v_row, q_batch, k_batch, v_batch;
  __nv_bfloat16* o;
  int64_t o_row, o_batch;
  float* lse;  // [B, Hq, Sq] base-2
  int B, Hq, Hkv, Sq, Sk;
  int q_offset, k_offset;
  int causal;
  float scale_log2;
};

// Load a [ROWS x D] tile (rows starting at r0 of a strided matrix) into swizzled smem.
template <int ROWS, int D, int NT>
__device__ __forceinline__ void load_tile(uint8_t* smem, const __nv_bfloat16* base, int64_t row_stride,
                                          int r0, int rmax) {
  constexpr int kChunks = ROWS * D / 8;
  for (int i = threadIdx.x; i < kChunks; i += NT) {
    const int r = i / (D / 8);
    const int c = (i % (D / 8)) * 8;
    const int gr = r0 + r;
    const bool ok = gr < rmax;
    const __nv_bfloat16* src = base + static_cast<int64_t>(ok ? gr : 0) * row_stride + c;
    cp_async16(smem + swz<D>(r, c), src, ok);
  }
}

// Forward: 128 query rows per CTA (8 warps x 16 rows), 64-key blocks, double buffered.
template <int D>
__global__ void __launch_bounds__(256) flash_fwd_kernel(const FwdParams p) {
  constexpr int BM = 128, BN = 64, NT = 256;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + BM * D * 2;
  uint8_t* sV = sK + 2 * BN * D * 2;

  const int mb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.Hq / p.Hkv);
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int m0 = mb * BM;

  const __nv_bfloat16* qb = p.q + b * p.q_batch + static_cast<int64_t>(h) * D;
  const __nv_bfloat16* kb = p.k + b * p.k_batch + static_cast<int64_t>(kvh) * D;
  const __nv_bfloat16* vb = p.v + b * p.v_batch + static_cast<int64_t>(kvh) * D;

  // Key range this query block can see.
  int n_end = p.Sk;
  if (p.causal) {
    const int last_q_pos = p.q_offset + min(m0 + BM, p.Sq) - 1;
    n_end = min(p.Sk, last_q_pos - p.k_offset + 1);
  }
  const int num_nb = n_end > 0 ? (n_end + BN - 1) / BN : 0;

  load_tile<BM, D, NT>(sQ, qb, p.q_row, m0, p.Sq);
  cp_async_commit();
  if (num_nb > 0) {
    load_tile<BN, D, NT>(sK, kb, p.k_row, 0, p.Sk);
    load_tile<BN, D, NT>(sV, vb, p.v_row, 0, p.Sk);
  }
  cp_async_commit();
  cp_async_wait<1>();
  __syncthreads();

  // Q fragments for this warp's 16 rows.
  uint32_t qf[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int c = kk * 16 + (lane >> 4) * 8;
    ldsm_x4(smem_u32(sQ) + swz<D>(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
  }

  float o_acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  const int qpos0 = p.q_offset + m0 + warp * 16 + g;  // row g; row g+8 is qpos0+8

  for (int nb = 0; nb < num_nb; ++nb) {
    const int buf = nb & 1;
    if (nb + 1 < num_nb) {
      load_tile<BN, D, NT>(sK + (buf ^ 1) * BN * D * 2, kb, p.k_row, (nb + 1) * BN, p.Sk);
      load_tile<BN, D, NT>(sV + (buf ^ 1) * BN * D * 2, vb, p.v_row, (nb + 1) * BN, p.Sk);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t kbase = smem_u32(sK + buf * BN * D * 2);
    const uint32_t vbase = smem_u32(sV + buf * BN * D * 2);

    float s[BN / 8][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int jp = 0; jp < BN / 16; ++jp) {
        uint32_t b0, b1, b2, b3;
        const int r = jp * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(kbase + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(s[2 * jp], qf[kk], b0, b1);
        mma_bf16(s[2 * jp + 1], qf[kk], b2, b3);
      }
    }
    // Scale, mask, online softmax.
    const int n0 = nb * BN;
    const bool need_mask = (n0 + BN > p.Sk) ||
                           (p.causal && (p.k_offset + n0 + BN - 1 > p.q_offset + m0 + warp * 16));
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[j][e] * p.scale_log2;
        if (need_mask) {
          const int kcol = n0 + j * 8 + 2 * t + (e & 1);
          const int qp = qpos0 + (e >> 1) * 8;
          if (kcol >= p.Sk || (p.causal && p.k_offset + kcol > qp)) x = -INFINITY;
        }
        s[j][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2], mnew[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mnew[r] = fmaxf(m_run[r], mx[r]);
      corr[r] = (m_run[r] == -INFINITY) ? 0.f : fast_exp2(m_run[r] - mnew[r]);
      if (mnew[r] == -INFINITY) corr[r] = 1.f;
      m_run[r] = mnew[r];
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pf[BN / 16][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = mnew[e >> 1];
        pv[e] = (mm == -INFINITY) ? 0.f : fast_exp2(s[j][e] - mm);
        rs[e >> 1] += pv[e];
      }
      pf[j >> 1][(j & 1) * 2 + 0] = pack_bf16x2(pv[0], pv[1]);
      pf[j >> 1][(j & 1) * 2 + 1] = pack_bf16x2(pv[2], pv[3]);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_run[r] = l_run[r] * corr[r] + rs[r];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o_acc[i][0] *= corr[0];
      o_acc[i][1] *= corr[0];
      o_acc[i][2] *= corr[1];
      o_acc[i][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dp * 16 + (lane >> 4) * 8;
        ldsm_x4_t(vbase + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(o_acc[2 * dp], a, b0, b1);
        mma_bf16(o_acc[2 * dp + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }

  // Finalise: full row sums, normalise, store O and LSE.
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  __nv_bfloat16* ob = p.o + b * p.o_batch + static_cast<int64_t>(h) * D;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = m0 + warp * 16 + g + r * 8;
    if (row >= p.Sq) continue;
    const float inv = l_run[r] > 0.f ? 1.f / l_run[r] : 0.f;
    __nv_bfloat16* orow = ob + static_cast<int64_t>(row) * p.o_row;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      *reinterpret_cast<uint32_t*>(orow + i * 8 + 2 * t) =
          pack_bf16x2(o_acc[i][2 * r] * inv, o_acc[i][2 * r + 1] * inv);
    }
    if (t == 0) {
      const float lse = l_run[r] > 0.f ? m_run[r] + __log2f(l_run[r]) : -INFINITY;
      p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.Sq + row] = lse;
    }
  }
}

// ------------------------------------------------------------------ backward
struct BwdParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const __nv_bfloat16* o;
  const __nv_bfloat16* dout;
  int64_t q_row, k_row, v_row, q_batch, k_batch, v_batch;
  int64_t o_row, o_batch, do_row, do_batch;
  const float* lse;    // [B, Hq, Sq]
  float* delta;        // [B, Hq, Sq]
  float* dq_acc;       // [B, Sq, Hq, D] fp32
  __nv_bfloat16* dq;   // output pointers (strided like q/k/v)
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int64_t dq_row, dk_row, dv_row, dq_batch, dk_batch, dv_batch;
  int B, Hq, Hkv, Sq, Sk;
  int q_offset, k_offset;
  int causal;
  float scale_log2;
  float scale;
  // optional inverse RoPE applied to dq / dk on the way out
  const int* q_pos;   // [Sq] or null
  const int* k_pos;   // [Sk] or null
  const float* inv_freq;
};

// delta = rowsum(dO * O); also zero the fp32 dQ accumulator. D / 8 threads per row, each
// with one 16-byte piece of O and dO; rows are ordered (b, h, s), which is the layout of
// delta, so a row's index is its delta index and a warp's delta stores are contiguous.
// The row's threads are consecutive lanes of one warp (D / 8 divides 32).
template <int D>
__global__ void __launch_bounds__(256) flash_bwd_pre_kernel(const BwdParams p) {
  constexpr int TPR = D / 8;
  const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t row = gt / TPR;
  const int part = static_cast<int>(gt % TPR);
  const bool ok = row < static_cast<int64_t>(p.B) * p.Hq * p.Sq;
  float acc = 0.f;
  if (ok) {
    const int s = static_cast<int>(row % p.Sq);
    const int h = static_cast<int>((row / p.Sq) % p.Hq);
    const int b = static_cast<int>(row / (static_cast<int64_t>(p.Sq) * p.Hq));
    const uint4 ov = __ldg(reinterpret_cast<const uint4*>(
        p.o + b * p.o_batch + static_cast<int64_t>(s) * p.o_row + h * D + part * 8));
    const uint4 dv = __ldg(reinterpret_cast<const uint4*>(
        p.dout + b * p.do_batch + static_cast<int64_t>(s) * p.do_row + h * D + part * 8));
    const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w}, dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e)
      acc += bf16_lo(ow[e]) * bf16_lo(dw[e]) + bf16_hi(ow[e]) * bf16_hi(dw[e]);
    float4* dqa = reinterpret_cast<float4*>(
        p.dq_acc + ((static_cast<int64_t>(b) * p.Sq + s) * p.Hq + h) * D + part * 8);
    dqa[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    dqa[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int off = TPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (ok && part == 0) p.delta[row] = acc;
}

template <int D>
static void launch_bwd_pre(const BwdParams& p, cudaStream_t stream) {
  const int64_t threads = static_cast<int64_t>(p.B) * p.Hq * p.Sq * (D / 8);
  flash_bwd_pre_kernel<D><<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(p);
}

__device__ __forceinline__ void red_add_v2(float* addr, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(addr), "f"(a), "f"(b) : "memory");
}

// Rotate-half inverse rotation of a pair (x1 at col c, x2 at col c + D/2).
__device__ __forceinline__ void inv_rope_pair(float& x1, float& x2, float ang) {
  float sn, cs;
  sincosf(ang, &sn, &cs);
  const float a = x1 * cs + x2 * sn;
  const float b = x2 * cs - x1 * sn;
  x1 = a;
  x2 = b;
}

template <int D>
__global__ void __launch_bounds__(128) flash_bwd_kernel(const BwdParams p) {
  constexpr int BM = 64, BN = 64, NT = 128;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sK = smem;
  uint8_t* sV = sK + BN * D * 2;
  uint8_t* sQ = sV + BN * D * 2;
  uint8_t* sdO = sQ + BM * D * 2;
  uint8_t* sdS = sdO + BM * D * 2;  // [BN kv rows x BM q cols] bf16, swizzled with D=BM
  float* sLse = reinterpret_cast<float*>(sdS + BN * BM * 2);
  float* sDelta = sLse + BM;

  const int nb = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int group = p.Hq / p.Hkv;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int n0 = nb * BN;

  const __nv_bfloat16* kb = p.k + b * p.k_batch + static_cast<int64_t>(kvh) * D;
  const __nv_bfloat16* vb = p.v + b * p.v_batch + static_cast<int64_t>(kvh) * D;
  load_tile<BN, D, NT>(sK, kb, p.k_row, n0, p.Sk);
  load_tile<BN, D, NT>(sV, vb, p.v_row, n0, p.Sk);
  cp_async_commit();

  float dk_acc[D / 8][4], dv_acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk_acc[i][e] = dv_acc[i][e] = 0.f;

  // First query block that can see this key block.
  int m_begin = 0;
  if (p.causal) {
    const int first_q = p.k_offset + n0 - p.q_offset;
    m_begin = max(0, first_q) / BM;
  }
  const int num_mb = (p.Sq + BM - 1) / BM;
  const int kv_row = n0 + warp * 16;  // this warp's first key row

  for (int hh = 0; hh < group; ++hh) {
    const int h = kvh * group + hh;
    const __nv_bfloat16* qb = p.q + b * p.q_batch + static_cast<int64_t>(h) * D;
    const __nv_bfloat16* dob = p.dout + b * p.do_batch + static_cast<int64_t>(h) * D;
    const float* lse_b = p.lse + (static_cast<int64_t>(b) * p.Hq + h) * p.Sq;
    const float* delta_b = p.delta + (static_cast<int64_t>(b) * p.Hq + h) * p.Sq;
    for (int mb = m_begin; mb < num_mb; ++mb) {
      const int m0 = mb * BM;
      __syncthreads();
      load_tile<BM, D, NT>(sQ, qb, p.q_row, m0, p.Sq);
      load_tile<BM, D, NT>(sdO, dob, p.do_row, m0, p.Sq);
      cp_async_commit();
      for (int i = threadIdx.x; i < BM; i += NT) {
        const int r = m0 + i;
        sLse[i] = r < p.Sq ? lse_b[r] : INFINITY;
        sDelta[i] = r < p.Sq ? delta_b[r] : 0.f;
      }
      cp_async_wait<0>();
      __syncthreads();
      const uint32_t kbase = smem_u32(sK), vbase = smem_u32(sV);
      const uint32_t qbase = smem_u32(sQ), dobase = smem_u32(sdO);

      // S^T = K Q^T (warp: 16 key rows x 64 query cols)
      float st[BM / 8][4];
      float dpt[BM / 8][4];
#pragma unroll
      for (int j = 0; j < BM / 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) st[j][e] = dpt[j][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t a[4], av[4];
        {
          const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = kk * 16 + (lane >> 4) * 8;
          ldsm_x4(kbase + swz<D>(r, c), a[0], a[1], a[2], a[3]);
          ldsm_x4(vbase + swz<D>(r, c), av[0], av[1], av[2], av[3]);
        }
#pragma unroll
        for (int jp = 0; jp < BM / 16; ++jp) {
          uint32_t b0, b1, b2, b3;
          const int r = jp * 16 + (lane & 7) + (lane >> 4) * 8;
          const int c = kk * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(qbase + swz<D>(r, c), b0, b1, b2, b3);
          mma_bf16(st[2 * jp], a, b0, b1);
          mma_bf16(st[2 * jp + 1], a, b2, b3);
          ldsm_x4(dobase + swz<D>(r, c), b0, b1, b2, b3);
          mma_bf16(dpt[2 * jp], av, b0, b1);
          mma_bf16(dpt[2 * jp + 1], av, b2, b3);
        }
      }
      // P^T and dS^T
      uint32_t pa[BM / 16][4], dsa[BM / 16][4];
#pragma unroll
      for (int j = 0; j < BM / 8; ++j) {
        float pv[4], dsv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int krow = kv_row + g + (e >> 1) * 8;
          const int qcol = j * 8 + 2 * t + (e & 1);
          const int qg = m0 + qcol;
          float pr = fast_exp2(st[j][e] * p.scale_log2 - sLse[qcol]);
          if (qg >= p.Sq || krow >= p.Sk || (p.causal && p.k_offset + krow > p.q_offset + qg))
            pr = 0.f;
          pv[e] = pr;
          dsv[e] = pr * (dpt[j][e] - sDelta[qcol]);
        }
        pa[j >> 1][(j & 1) * 2 + 0] = pack_bf16x2(pv[0], pv[1]);
        pa[j >> 1][(j & 1) * 2 + 1] = pack_bf16x2(pv[2], pv[3]);
        dsa[j >> 1][(j & 1) * 2 + 0] = pack_bf16x2(dsv[0], dsv[1]);
        dsa[j >> 1][(j & 1) * 2 + 1] = pack_bf16x2(dsv[2], dsv[3]);
        // stash dS^T (bf16) for the dQ product
        const int r0 = warp * 16 + g;
        const int c0 = j * 8 + 2 * t;
        *reinterpret_cast<uint32_t*>(sdS + swz<BM>(r0, c0)) = dsa[j >> 1][(j & 1) * 2 + 0];
        *reinterpret_cast<uint32_t*>(sdS + swz<BM>(r0 + 8, c0)) = dsa[j >> 1][(j & 1) * 2 + 1];
      }
      // dV += P^T dO ; dK += dS^T Q
#pragma unroll
      for (int kk = 0; kk < BM / 16; ++kk) {
#pragma unroll
        for (int dp = 0; dp < D / 16; ++dp) {
          uint32_t b0, b1, b2, b3;
          const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = dp * 16 + (lane >> 4) * 8;
          ldsm_x4_t(dobase + swz<D>(r, c), b0, b1, b2, b3);
          mma_bf16(dv_acc[2 * dp], pa[kk], b0, b1);
          mma_bf16(dv_acc[2 * dp + 1], pa[kk], b2, b3);
          ldsm_x4_t(qbase + swz<D>(r, c), b0, b1, b2, b3);
          mma_bf16(dk_acc[2 * dp], dsa[kk], b0, b1);
          mma_bf16(dk_acc[2 * dp + 1], dsa[kk], b2, b3);
        }
      }
      __syncthreads();
      // dQ[q rows of this warp] += dS K, in two halves of D to bound registers.
      const uint32_t dsbase = smem_u32(sdS);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float dq[D / 16][4];
#pragma unroll
        for (int i = 0; i < D / 16; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          uint32_t a[4];
          {
            const int r = kk * 16 + (lane & 7) + (lane >> 4) * 8;       // kv row
            const int c = warp * 16 + ((lane >> 3) & 1) * 8;            // q col
            ldsm_x4_t(dsbase + swz<BM>(r, c), a[0], a[1], a[2], a[3]);
          }
#pragma unroll
          for (int dp = 0; dp < D / 32; ++dp) {
            uint32_t b0, b1, b2, b3;
            const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
            const int c = half * (D / 2) + dp * 16 + (lane >> 4) * 8;
            ldsm_x4_t(kbase + swz<D>(r, c), b0, b1, b2, b3);
            mma_bf16(dq[2 * dp], a, b0, b1);
            mma_bf16(dq[2 * dp + 1], a, b2, b3);
          }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int qrow = m0 + warp * 16 + g + r * 8;
          if (qrow >= p.Sq) continue;
          float* dst = p.dq_acc + ((static_cast<int64_t>(b) * p.Sq + qrow) * p.Hq + h) * D +
                       half * (D / 2);
#pragma unroll
          for (int i = 0; i < D / 16; ++i)
            red_add_v2(dst + i * 8 + 2 * t, dq[i][2 * r] * p.scale, dq[i][2 * r + 1] * p.scale);
        }
      }
    }
  }

  // Store dK (with optional inverse RoPE) and dV for this warp's 16 key rows.
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int krow = kv_row + g + r * 8;
    if (krow >= p.Sk) continue;
    if (p.k_pos != nullptr) {
      const float pos = static_cast<float>(__ldg(p.k_pos + krow));
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int c = i * 8 + 2 * t + e;  // c < D/2
          float x1 = dk_acc[i][2 * r + e], x2 = dk_acc[i + D / 16][2 * r + e];
          inv_rope_pair(x1, x2, pos * __ldg(p.inv_freq + c));
          dk_acc[i][2 * r + e] = x1;
          dk_acc[i + D / 16][2 * r + e] = x2;
        }
      }
    }
    __nv_bfloat16* dkr = p.dk + b * p.dk_batch + static_cast<int64_t>(krow) * p.dk_row +
                         static_cast<int64_t>(kvh) * D;
    __nv_bfloat16* dvr = p.dv + b * p.dv_batch + static_cast<int64_t>(krow) * p.dv_row +
                         static_cast<int64_t>(kvh) * D;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      *reinterpret_cast<uint32_t*>(dkr + i * 8 + 2 * t) =
          pack_bf16x2(dk_acc[i][2 * r] * p.scale, dk_acc[i][2 * r + 1] * p.scale);
      *reinterpret_cast<uint32_t*>(dvr + i * 8 + 2 * t) =
          pack_bf16x2(dv_acc[i][2 * r], dv_acc[i][2 * r + 1]);
    }
  }
}

// dq_acc (fp32) -> dq (bf16) with optional inverse RoPE. One thread per pair.
// dq = bf16(dq_acc), with the inverse rotate-half RoPE when positions are given. A thread
// takes 8 rotation pairs (columns c..c+7 and c+D/2..c+D/2+7) of up to 4 heads of one
// (b, s) row: the angles depend only on the position and the pair, so each thread
// evaluates 8 sincosf and reuses them across its heads. 16-byte loads and stores.
constexpr int kDqHeadsPerThread = 4;

template <int D>
__global__ void __launch_bounds__(256) flash_bwd_dq_kernel(const BwdParams p) {
  constexpr int CH = D / 16;  // 8-pair chunks per head
  const int hgroups = (p.Hq + kDqHeadsPerThread - 1) / kDqHeadsPerThread;
  const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gt >= static_cast<int64_t>(p.B) * p.Sq * hgroups * CH) return;
  const int j = static_cast<int>(gt % CH);
  const int hg = static_cast<int>((gt / CH) % hgroups);
  const int64_t bs = gt / (static_cast<int64_t>(CH) * hgroups);
  const int s = static_cast<int>(bs % p.Sq);
  const int b = static_cast<int>(bs / p.Sq);
  const bool rope = p.q_pos != nullptr;
  float cs[8], sn[8];
  if (rope) {
    const float pos = static_cast<float>(__ldg(p.q_pos + s));
#pragma unroll
    for (int e = 0; e < 8; ++e) sincosf(pos * __ldg(p.inv_freq + j * 8 + e), &sn[e], &cs[e]);
  }
  const int h0 = hg * kDqHeadsPerThread, h1 = min(p.Hq, h0 + kDqHeadsPerThread);
  const float* src = p.dq_acc + bs * p.Hq * D + j * 8;
  __nv_bfloat16* dst = p.dq + b * p.dq_batch + static_cast<int64_t>(s) * p.dq_row + j * 8;
#pragma unroll 2
  for (int h = h0; h < h1; ++h) {
    const float4* a4 = reinterpret_cast<const float4*>(src + h * D);
    const float4* b4 = reinterpret_cast<const float4*>(src + h * D + D / 2);
    const float4 a0 = a4[0], a1 = a4[1], b0 = b4[0], b1 = b4[1];
    float x1[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    float x2[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    if (rope) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float u = x1[e] * cs[e] + x2[e] * sn[e];
        const float w = x2[e] * cs[e] - x1[e] * sn[e];
        x1[e] = u;
        x2[e] = w;
      }
    }
    *reinterpret_cast<uint4*>(dst + h * D) =
        make_uint4(pack_bf16x2(x1[0], x1[1]), pack_bf16x2(x1[2], x1[3]),
                   pack_bf16x2(x1[4], x1[5]), pack_bf16x2(x1[6], x1[7]));
    *reinterpret_cast<uint4*>(dst + h * D + D / 2) =
        make_uint4(pack_bf16x2(x2[0], x2[1]), pack_bf16x2(x2[2], x2[3]),
                   pack_bf16x2(x2[4], x2[5]), pack_bf16x2(x2[6], x2[7]));
  }
}

template <int D>
static void launch_bwd_dq(const BwdParams& p, cudaStream_t stream) {
  const int64_t threads = static_cast<int64_t>(p.B) * p.Sq *
                          ((p.Hq + kDqHeadsPerThread - 1) / kDqHeadsPerThread) * (D / 16);
  flash_bwd_dq_kernel<D><<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(p);
}

}  // namespace attn
}  // namespace nmb

using namespace nmb;
using namespace nmb::attn;

static void check_rows(const at::Tensor& t, const char* name, int64_t D) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, name, " must be CUDA bf16");
  TORCH_CHECK(t.dim() == 4, name, " must be [B, S, H, D]");
  TORCH_CHECK(t.size(3) == D && t.stride(3) == 1 && t.stride(2) == D, name,
              " must have contiguous heads");
  TORCH_CHECK(t.stride(1) % 8 == 0 && t.stride(0) % 8 == 0, name, " strides must be 16-byte");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
}

// q: [B, Sq, Hq, D], k/v: [B, Sk, Hkv, D] (strided views), o: [B, Sq, Hq, D], lse: [B, Hq, Sq] f32
void flash_attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse,
                    double softmax_scale, bool causal, int64_t q_offset, int64_t k_offset) {
  const int64_t D = q.size(3);
  TORCH_CHECK(D == 64 || D == 128, "flash_attn_fwd: head_dim must be 64 or 128");
  check_rows(q, "q", D);
  check_rows(k, "k", D);
  check_rows(v, "v", D);
  check_rows(o, "o", D);
  FwdParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  p.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.q_row = q.stride(1);
  p.q_batch = q.stride(0);
  p.k_row = k.stride(1);
  p.k_batch = k.stride(0);
  p.v_row = v.stride(1);
  p.v_batch = v.stride(0);
  p.o_row = o.stride(1);
  p.o_batch = o.stride(0);
  p.lse = lse.data_ptr<float>();
  p.B = q.size(0);
  p.Sq = q.size(1);
  p.Hq = q.size(2);
  p.Sk = k.size(1);
  p.Hkv = k.size(2);
  TORCH_CHECK(p.Hq % p.Hkv == 0, "query heads must be a multiple of kv heads");
  p.q_offset = q_offset;
  p.k_offset = k_offset;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = static_cast<float>(softmax_scale) * kLog2e;
  if (p.B == 0 || p.Sq == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  dim3 grid((p.Sq + 127) / 128, p.Hq, p.B);
  if (D == 64) {
    const int smem = (128 + 4 * 64) * 64 * 2;
    auto kern = flash_fwd_kernel<64>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<grid, 256, smem, stream>>>(p); NMB_LAUNCHED(1);
  } else {
    const int smem = (128 + 4 * 64) * 128 * 2;
    auto kern = flash_fwd_kernel<128>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<grid, 256, smem, stream>>>(p); NMB_LAUNCHED(1);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Backward. dq/dk/dv are [B, S, H, D] strided views (typically slices of one
// fused dQKV buffer). `q_pos`/`k_pos` (int32 positions) + `inv_freq` enable the
// fused inverse RoPE on dq/dk.
void flash_attn_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor dout,
                    at::Tensor lse, at::Tensor dq, at::Tensor dk, at::Tensor dv,
                    at::Tensor delta_ws, at::Tensor dq_acc_ws, double softmax_scale, bool causal,
                    int64_t q_offset, int64_t k_offset, c10::optional<at::Tensor> q_pos,
                    c10::optional<at::Tensor> k_pos, c10::optional<at::Tensor> inv_freq) {
  const int64_t D = q.size(3);
  TORCH_CHECK(D == 64 || D == 128, "flash_attn_bwd: head_dim must be 64 or 128");
  check_rows(q, "q", D);
  check_rows(k, "k", D);
  check_rows(v, "v", D);
  check_rows(o, "o", D);
  check_rows(dout, "dout", D);
  check_rows(dq, "dq", D);
  check_rows(dk, "dk", D);
  check_rows(dv, "dv", D);
  BwdParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  p.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  p.o = reinterpret_cast<const __nv_bfloat16*>(o.data_ptr());
  p.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  p.q_row = q.stride(1);
  p.q_batch = q.stride(0);
  p.k_row = k.stride(1);
  p.k_batch = k.stride(0);
  p.v_row = v.stride(1);
  p.v_batch = v.stride(0);
  p.o_row = o.stride(1);
  p.o_batch = o.stride(0);
  p.do_row = dout.stride(1);
  p.do_batch = dout.stride(0);
  p.lse = lse.data_ptr<float>();
  p.B = q.size(0);
  p.Sq = q.size(1);
  p.Hq = q.size(2);
  p.Sk = k.size(1);
  p.Hkv = k.size(2);
  TORCH_CHECK(delta_ws.numel() >= static_cast<int64_t>(p.B) * p.Hq * p.Sq, "delta workspace too small");
  TORCH_CHECK(dq_acc_ws.numel() >= static_cast<int64_t>(p.B) * p.Hq * p.Sq * D,
              "dq accumulator workspace too small");
  p.delta = delta_ws.data_ptr<float>();
  p.dq_acc = dq_acc_ws.data_ptr<float>();
  p.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.dq_row = dq.stride(1);
  p.dq_batch = dq.stride(0);
  p.dk_row = dk.stride(1);
  p.dk_batch = dk.stride(0);
  p.dv_row = dv.stride(1);
  p.dv_batch = dv.stride(0);
  p.q_offset = q_offset;
  p.k_offset = k_offset;
  p.causal = causal ? 1 : 0;
  p.scale = static_cast<float>(softmax_scale);
  p.scale_log2 = static_cast<float>(softmax_scale) * kLog2e;
  p.q_pos = q_pos.has_value() ? q_pos->data_ptr<int>() : nullptr;
  p.k_pos = k_pos.has_value() ? k_pos->data_ptr<int>() : nullptr;
  p.inv_freq = inv_freq.has_value() ? inv_freq->data_ptr<float>() : nullptr;
  TORCH_CHECK((p.q_pos == nullptr && p.k_pos == nullptr) || p.inv_freq != nullptr,
              "inverse RoPE needs inv_freq");
  if (p.B == 0 || p.Sq == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  dim3 grid((p.Sk + 63) / 64, p.Hkv, p.B);
  if (D == 64) {
    launch_bwd_pre<64>(p, stream); NMB_LAUNCHED(1);
    const int smem = (4 * 64 * 64 + 64 * 64) * 2 + 2 * 64 * 4;
    auto kern = flash_bwd_kernel<64>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<grid, 128, smem, stream>>>(p); NMB_LAUNCHED(1);
    launch_bwd_dq<64>(p, stream); NMB_LAUNCHED(1);
  } else {
    launch_bwd_pre<128>(p, stream); NMB_LAUNCHED(1);
    const int smem = (4 * 64 * 128 + 64 * 64) * 2 + 2 * 64 * 4;
    auto kern = flash_bwd_kernel<128>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<grid, 128, smem, stream>>>(p); NMB_LAUNCHED(1);
    launch_bwd_dq<128>(p, stream); NMB_LAUNCHED(1);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the backward (declared and documented in noalloc.h).
// Same three kernels as flash_attn_bwd above; its two temporaries live in a
// fixed device array owned by this file instead of caller-provided workspaces.
#include <mutex>

#include "noalloc.h"

namespace nmb {
namespace attn {

static __device__ __align__(256) float g_noalloc_scratch[NMB_NOALLOC_SCRATCH_FLOATS];

constexpr int kNoAllocMaxDevices = 64;
static float* g_noalloc_scratch_addr[kNoAllocMaxDevices] = {nullptr};
static std::mutex g_noalloc_mutex;

// Device address of the scratch array for the current device (set up once).
static float* noalloc_scratch_for_current_device(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) {
    *err = NMB_NOALLOC_SETUP_FAILED;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_scratch_addr[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (rc != cudaSuccess || ptr == nullptr) {
      *err = NMB_NOALLOC_SETUP_FAILED;
      return nullptr;
    }
    g_noalloc_scratch_addr[dev] = static_cast<float*>(ptr);
  }
  return g_noalloc_scratch_addr[dev];
}

template <int D>
static int noalloc_launch(const BwdParams& p, cudaStream_t stream) {
  const int smem = (4 * 64 * D + 64 * 64) * 2 + 2 * 64 * 4;
  if (cudaFuncSetAttribute(flash_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           smem) != cudaSuccess)
    return NMB_NOALLOC_LAUNCH_FAILED;
  // An error left pending by some earlier, unrelated call is not this call's failure:
  // clear it first, so the check after each launch below sees only our own launches.
  (void)cudaGetLastError();
  dim3 grid((p.Sk + 63) / 64, p.Hkv, p.B);
  // pre: delta = rowsum(dO * O) and dq_acc = 0; the main kernel adds into dq_acc; dq:
  // dq = bf16(dq_acc). With no keys (Sk == 0) the main kernel has nothing to do and dq
  // comes out as zeros.
  launch_bwd_pre<D>(p, stream);
  if (cudaGetLastError() != cudaSuccess) return NMB_NOALLOC_LAUNCH_FAILED;
  int launched = 1;
  if (p.Sk > 0) {
    flash_bwd_kernel<D><<<grid, 128, smem, stream>>>(p);
    if (cudaGetLastError() != cudaSuccess) return NMB_NOALLOC_LAUNCH_FAILED;
    ++launched;
  }
  launch_bwd_dq<D>(p, stream);
  if (cudaGetLastError() != cudaSuccess) return NMB_NOALLOC_LAUNCH_FAILED;
  NMB_LAUNCHED(launched + 1);
  return NMB_NOALLOC_OK;
}

}  // namespace attn
}  // namespace nmb

extern "C" int nmb_flash_attn_bwd_noalloc(const void* q, const void* k, const void* v,
                                          const void* o, const void* dout, const float* lse,
                                          void* dq, void* dk, void* dv, int batch, int seq_q,
                                          int seq_k, int heads_q, int heads_kv, int head_dim,
                                          float softmax_scale, int causal, int q_offset,
                                          int k_offset, cudaStream_t stream) {
  using namespace nmb::attn;
  const void* ptrs[] = {q, k, v, o, dout, lse, dq, dk, dv};
  for (const void* ptr : ptrs)
    if (ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 15u) != 0)
      return NMB_NOALLOC_BAD_ARGUMENT;
  if ((head_dim != 64 && head_dim != 128) || batch < 0 || seq_q < 0 || seq_k < 0 ||
      heads_q <= 0 || heads_kv <= 0 || heads_q % heads_kv != 0)
    return NMB_NOALLOC_BAD_ARGUMENT;
  const long long rows = static_cast<long long>(batch) * seq_q * heads_q;
  const long long delta_floats = (rows + 63) / 64 * 64;  // keeps dq_acc 256-byte aligned
  if (delta_floats + rows * head_dim > NMB_NOALLOC_SCRATCH_FLOATS) return NMB_NOALLOC_TOO_LARGE;
  if (rows == 0) return NMB_NOALLOC_OK;
  int err = NMB_NOALLOC_OK;
  float* scratch = noalloc_scratch_for_current_device(&err);
  if (scratch == nullptr) return err;

  BwdParams p{};
  const int64_t D = head_dim;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.o = static_cast<const __nv_bfloat16*>(o);
  p.dout = static_cast<const __nv_bfloat16*>(dout);
  p.q_row = p.o_row = p.do_row = p.dq_row = heads_q * D;
  p.q_batch = p.o_batch = p.do_batch = p.dq_batch = static_cast<int64_t>(seq_q) * heads_q * D;
  p.k_row = p.v_row = p.dk_row = p.dv_row = heads_kv * D;
  p.k_batch = p.v_batch = p.dk_batch = p.dv_batch = static_cast<int64_t>(seq_k) * heads_kv * D;
  p.lse = lse;
  p.delta = scratch;
  p.dq_acc = scratch + delta_floats;
  p.dq = static_cast<__nv_bfloat16*>(dq);
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  p.B = batch;
  p.Sq = seq_q;
  p.Sk = seq_k;
  p.Hq = heads_q;
  p.Hkv = heads_kv;
  p.q_offset = q_offset;
  p.k_offset = k_offset;
  p.causal = causal ? 1 : 0;
  p.scale = softmax_scale;
  p.scale_log2 = softmax_scale * kLog2e;
  return head_dim == 64 ? noalloc_launch<64>(p, stream) : noalloc_launch<128>(p, stream);
}

extern "C" const char* nmb_noalloc_strerror(int code) {
  switch (code) {
    case NMB_NOALLOC_OK: return "ok";
    case NMB_NOALLOC_BAD_ARGUMENT:
      return "bad argument: null or non-16-byte-aligned pointer, head_dim not 64/128, or "
             "heads_q not a multiple of heads_kv";
    case NMB_NOALLOC_TOO_LARGE:
      return "problem too large for the fixed scratch: needs B*Hq*Sq*(D+1) floats (+64) <= "
             "NMB_NOALLOC_SCRATCH_FLOATS (8 Mi floats)";
    case NMB_NOALLOC_SETUP_FAILED:
      return "could not resolve the scratch array's device address on the current device";
    case NMB_NOALLOC_LAUNCH_FAILED: return "kernel launch failed";
    default: return "unknown error";
  }
}

// ---------------------------------------------------------------------------
// Stand-alone pieces of the backward used with the tcgen05 dK/dV/dQ kernel
// (attention_tc_bwd.cu): preparation (delta = rowsum(dO * O), zero the fp32 dQ
// accumulator) and the final dQ conversion (with optional inverse RoPE).
static BwdParams prep_params(const at::Tensor& o, const at::Tensor& dout, at::Tensor& delta,
                             at::Tensor& dq_acc) {
  BwdParams p{};
  p.o = reinterpret_cast<const __nv_bfloat16*>(o.data_ptr());
  p.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  p.o_row = o.stride(1);
  p.o_batch = o.stride(0);
  p.do_row = dout.stride(1);
  p.do_batch = dout.stride(0);
  p.B = o.size(0);
  p.Sq = o.size(1);
  p.Hq = o.size(2);
  p.delta = delta.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  return p;
}

void flash_attn_bwd_prep(at::Tensor o, at::Tensor dout, at::Tensor delta, at::Tensor dq_acc) {
  const int64_t D = o.size(3);
  TORCH_CHECK(D == 64 || D == 128);
  check_rows(o, "o", D);
  check_rows(dout, "dout", D);
  BwdParams p = prep_params(o, dout, delta, dq_acc);
  TORCH_CHECK(delta.numel() >= static_cast<int64_t>(p.B) * p.Hq * p.Sq);
  TORCH_CHECK(dq_acc.numel() >= static_cast<int64_t>(p.B) * p.Hq * p.Sq * D);
  if (p.B == 0 || p.Sq == 0) return;
  const at::cuda::CUDAGuard guard(o.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (D == 64)
    launch_bwd_pre<64>(p, stream);
  else
    launch_bwd_pre<128>(p, stream);
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void flash_attn_bwd_dq_convert(at::Tensor dq_acc, at::Tensor dq, c10::optional<at::Tensor> q_pos,
                               c10::optional<at::Tensor> inv_freq) {
  const int64_t D = dq.size(3);
  TORCH_CHECK(D == 64 || D == 128);
  check_rows(dq, "dq", D);
  BwdParams p{};
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  p.dq_row = dq.stride(1);
  p.dq_batch = dq.stride(0);
  p.B = dq.size(0);
  p.Sq = dq.size(1);
  p.Hq = dq.size(2);
  p.q_pos = q_pos.has_value() ? q_pos->data_ptr<int>() : nullptr;
  p.inv_freq = inv_freq.has_value() ? inv_freq->data_ptr<float>() : nullptr;
  TORCH_CHECK(p.q_pos == nullptr || p.inv_freq != nullptr);
  if (p.B == 0 || p.Sq == 0) return;
  const at::cuda::CUDAGuard guard(dq.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (D == 64)
    launch_bwd_dq<64>(p, stream);
  else
    launch_bwd_dq<128>(p, stream);
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Causal flash-attention backward on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// One CTA per (128-key block, KV head, batch); it loops over the query heads of
// its GQA group and over the 128-query blocks that can see its keys. Per query
// block, with K, V resident in shared memory:
//   MMA  : S^T = K Q^T and dP^T = V dO^T            -> TMEM cols [0,128) / [128,256)
//   warps: each thread owns one key row; P^T = exp2(S^T*c - lse), dS^T =
//          P^T (dP^T - delta) -> bf16 tiles in shared memory (UMMA SW128 layout)
//   MMA  : dV += P^T dO ; dK += dS^T Q                -> TMEM (resident accumulators)
//          dQ  = dS K                                  -> TMEM cols [0, D) (reuses S^T)
//   warps: each thread owns one query row of dQ and adds it (x softmax scale)
//          into the fp32 dQ accumulator in global memory with vector reductions.
// At the end dK (x scale, inverse RoPE when positions are given) and dV are
// written as bf16. The dQ accumulator is prepared (zeroed, delta = rowsum(dO*O))
// and converted (with inverse RoPE) by the helper kernels of attention.cu.
//
// Operand layouts (all 128-byte swizzled, loaded by TMA): K/Q/dO/V tiles serve
// as K-major operands for S^T / dP^T and as MN-major operands for dV / dK / dQ;
// the P^T / dS^T tiles are K-major A for dV / dK and MN-major A for dQ.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>

#include <cstdlib>

#include "common.cuh"

namespace nmb {
namespace fabw {

constexpr int kBN = 128;  // keys per CTA
constexpr int kBM = 128;  // queries per step
// Threads: warp 0 loads (TMA), warp 1 issues the MMAs, then SH groups of four
// softmax warps. With SH = 2 the two groups split the 128 query columns of each
// step (and the dQ / dK-dV drains) in halves: warp w reads TMEM lane quarter w % 4.
// The last warp pulls the next ring step's K/V block (context parallelism; idle otherwise).
template <int SH>
constexpr int threads_for() { return 64 + 128 * SH + 32; }
template <int SH>
constexpr int pull_warp() { return 2 + 4 * SH; }
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct Cfg {
  // D = 64 runs pipelined: Q/dO double-buffered in shared memory and dQ in its own TMEM
  // columns, so the next step's loads and S^T/dP^T MMAs overlap this step's dQ drain.
  // D = 128 has neither the shared memory nor the TMEM for that and runs step by step.
  static constexpr bool kPipe = D == 64;
  static constexpr int kQStages = kPipe ? 2 : 1;
  static constexpr int kTile = 128 * D * 2;             // one 128-row bf16 tile
  static constexpr int kPTile = kBN * kBM * 2;           // P^T or dS^T
  static constexpr int kSmem =
      (2 + 2 * kQStages) * kTile + 2 * kPTile + 2 * kBM * 4 + 1024 + 256;
  static constexpr int kTmemCols = 512;
  // TMEM columns: S^T [0,128), dP^T [128,256), dV [256, 256+D), dK [256+D, 256+2D);
  // dQ at [384, 448) when pipelined (D = 64), else it reuses S^T's [0, D).
  static constexpr int kColS = 0, kColDP = 128, kColDV = 256, kColDK = 256 + D;
  static constexpr int kColDQ = kPipe ? 384 : 0;
};

struct Params {
  const float* lse;     // [B, Hq, Sq] base 2
  const float* delta;   // [B, Hq, Sq]
  float* dq_acc;        // [B, Sq, Hq, D], or [key blocks][B, Sq, Hq, D] (dq_slot_stride)
  // 0: dQ partials are added into dq_acc with fp32 atomics. > 0 (deterministic mode): key
  // block nb stores its partial into slot nb (dq_acc + nb * dq_slot_stride, zeroed by the
  // caller) with plain stores, and the caller sums the slots in order.
  int64_t dq_slot_stride;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int64_t dk_row, dk_batch, dv_row, dv_batch;
  int B, Hq, Hkv, Sq, Sk;
  int q_offset, k_offset;
  int causal;
  float scale_log2, scale;
  const int* k_pos;
  const float* inv_freq;
  const float2* k_cs;   // optional (cos, sin)(k_pos[row] * inv_freq[i]) table [Sk][D/2]
  // optional phase trace: kTraceSlots %globaltimer stamps per CTA (see kTrace* below)
  unsigned long long* trace;
  int* status;
  PullDesc pull;
};

// Phase trace layout per CTA (nanoseconds, %globaltimer): [0] entry, [1] set-up done,
// [2] end of the dK/dV epilogue; softmax thread, for the first kTraceSteps steps t:
// [3 + 6t + e] e = 0 step start, 1 S/dP ready, 2 P/dS tiles free, 3 P/dS written,
// 4 dV/dK/dQ done, 5 dQ drained; MMA thread: [3 + 6 kTraceSteps + 2t + e] e = 0 Q/dO
// landed, 1 P/dS ready. Written only when Params::trace is set (a diagnostic run).
// [3 + 8 kTraceSteps + e]: inside step 0's first P/dS chunk, e = 0 TMEM loads landed,
// 1 values computed, 2 tiles stored; e = 3 all chunks done.
constexpr int kTraceSteps = 5;
constexpr int kTraceChunk = 3 + 8 * kTraceSteps;
constexpr int kTraceSlots = kTraceChunk + 4;

__device__ __forceinline__ void trace_stamp(const Params& p, int slot) {
  if (p.trace != nullptr)
    p.trace[(blockIdx.x + static_cast<long long>(gridDim.x) * blockIdx.y) * kTraceSlots + slot] =
        globaltimer_ns();
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const void* desc, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

// Write 32 bf16 values (16 packed pairs) = columns [32c, 32c+32) of row `row` into a
// [128 rows x 128 cols] SW128 tile (two 64-column swizzle atoms).
__device__ __forceinline__ void store_chunk_sw128(uint8_t* tile, int row, int c,
                                                  const uint32_t* pk) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int ch = c * 4 + q;
    const int atom = ch >> 3, c8 = ch & 7;
    uint8_t* dst = tile + atom * (128 * 128) + row * 128 + ((c8 ^ (row & 7)) << 4);
    *reinterpret_cast<uint4*>(dst) = make_uint4(pk[q * 4], pk[q * 4 + 1], pk[q * 4 + 2],
                                                pk[q * 4 + 3]);
  }
}

// Write a 128-value bf16 row (packed pairs) into a [128 rows x 128 cols] SW128 tile.
__device__ __forceinline__ void store_row_sw128(uint8_t* tile, int row, const uint32_t* pk) {
#pragma unroll
  for (int ch = 0; ch < 16; ++ch) {
    const int atom = ch >> 3, c8 = ch & 7;
    uint8_t* dst = tile + atom * (128 * 128) + row * 128 + ((c8 ^ (row & 7)) << 4);
    *reinterpret_cast<uint4*>(dst) = make_uint4(pk[ch * 4], pk[ch * 4 + 1], pk[ch * 4 + 2],
                                                pk[ch * 4 + 3]);
  }
}

template <int D, int SH>
__global__ void __launch_bounds__(threads_for<SH>(), 1)
    flash_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmDO, const Params p) {
  using C = Cfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  constexpr int QS = C::kQStages;
  uint8_t* sK = smem;
  uint8_t* sV = sK + C::kTile;
  uint8_t* sQ0 = sV + C::kTile;                  // QS stages of Q, then QS stages of dO
  uint8_t* sDO0 = sQ0 + QS * C::kTile;
  uint8_t* sP = sDO0 + QS * C::kTile;
  uint8_t* sDS = sP + C::kPTile;
  float* sLse = reinterpret_cast<float*>(sDS + C::kPTile);
  float* sDelta = sLse + kBM;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDelta + kBM);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;   // [QS]
  uint64_t* qdo_empty = bars + 3;  // [QS]
  uint64_t* sdp_full = bars + 5;   // S^T and dP^T in TMEM
  uint64_t* pds_full = bars + 6;   // P^T and dS^T in smem (4 * SH warp arrivals)
  uint64_t* mm_done = bars + 7;    // dV/dK/dQ MMAs of a step complete
  uint64_t* dq_free = bars + 8;    // dQ drained from TMEM (4 * SH warp arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // Key block is the slowest grid index: the (causally) longest CTAs, key block 0,
  // start first, which shortens the tail of the launch.
  const int nb = blockIdx.y, kvh = blockIdx.x % p.Hkv, b = blockIdx.x / p.Hkv;
  const int group = p.Hq / p.Hkv;
  const int n0 = nb * kBN;
  const int warp = threadIdx.x / 32;
  int m_begin = 0;
  if (p.causal) m_begin = max(0, p.k_offset + n0 - p.q_offset) / kBM;
  const int num_mb = (p.Sq + kBM - 1) / kBM;
  const int steps_per_head = max(0, num_mb - m_begin);
  const int total_steps = steps_per_head * group;

  if (threadIdx.x == 64) trace_stamp(p, 0);
  if (threadIdx.x == 0) {
    for (int i = 0; i < 9; ++i) mbar_init(&bars[i], (i == 6 || i == 8) ? 4 * SH : 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 64) trace_stamp(p, 1);

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (elect_one() && total_steps > 0) {
      mbar_arrive_expect_tx(kv_full, 2 * C::kTile);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_4d(sK + c * 128 * 128, &tmK, kv_full, c * 64, kvh, n0, b);
        tma_load_4d(sV + c * 128 * 128, &tmV, kv_full, c * 64, kvh, n0, b);
      }
      for (int t = 0; t < total_steps; ++t) {
        const int h = kvh * group + t / steps_per_head;
        const int m0 = (m_begin + t % steps_per_head) * kBM;
        const int st = t % QS;
        const uint32_t ph = static_cast<uint32_t>(t / QS) & 1u;
        if (!mbar_wait(&qdo_empty[st], ph ^ 1u, p.status, kStatusAttnTimeout, abort_flag)) break;
        mbar_arrive_expect_tx(&qdo_full[st], 2 * C::kTile);
        uint8_t* sQ = sQ0 + st * C::kTile;
        uint8_t* sDO = sDO0 + st * C::kTile;
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(sQ + c * 128 * 128, &tmQ, &qdo_full[st], c * 64, h, m0, b);
          tma_load_4d(sDO + c * 128 * 128, &tmDO, &qdo_full[st], c * 64, h, m0, b);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (elect_one() && total_steps > 0) {
      constexpr uint32_t id_s = umma_idesc_bf16(kBN, kBM, false, false);  // K-major A, B
      constexpr uint32_t id_acc = umma_idesc_bf16(kBN, D, false, true);   // dV, dK
      constexpr uint32_t id_dq = umma_idesc_bf16(kBM, D, true, true);     // dQ
      bool ok = mbar_wait(kv_full, 0, p.status, kStatusAttnTimeout, abort_flag);
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP),
                     aDS = smem_u32(sDS);
      for (int t = 0; t < total_steps && ok; ++t) {
        const int st = t % QS;
        const uint32_t aQ = smem_u32(sQ0 + st * C::kTile), aDO = smem_u32(sDO0 + st * C::kTile);
        ok = mbar_wait(&qdo_full[st], static_cast<uint32_t>(t / QS) & 1u, p.status,
                       kStatusAttnTimeout, abort_flag);
        if (t < kTraceSteps) trace_stamp(p, 3 + 6 * kTraceSteps + 2 * t);
        // Unpipelined: S^T shares TMEM with the previous step's dQ, which must be drained.
        if (ok && !C::kPipe && t > 0)
          ok = mbar_wait(dq_free, (t - 1) & 1, p.status, kStatusAttnTimeout, abort_flag);
        if (!ok) break;
        tc_fence_after();
        // S^T = K Q^T ; dP^T = V dO^T   (M = keys, N = queries, K = D)
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem + C::kColS, umma_desc_sw128(aK + off, 16, 1024),
                      umma_desc_sw128(aQ + off, 16, 1024), id_s, kk > 0);
          umma_f16_ss(tmem + C::kColDP, umma_desc_sw128(aV + off, 16, 1024),
                      umma_desc_sw128(aDO + off, 16, 1024), id_s, kk > 0);
        }
        umma_commit(sdp_full);
        ok = mbar_wait(pds_full, t & 1, p.status, kStatusAttnTimeout, abort_flag);
        if (t < kTraceSteps) trace_stamp(p, 3 + 6 * kTraceSteps + 2 * t + 1);
        // Pipelined: the previous dQ (own columns) must be drained before this step's dQ.
        if (ok && C::kPipe && t > 0)
          ok = mbar_wait(dq_free, (t - 1) & 1, p.status, kStatusAttnTimeout, abort_flag);
        if (!ok) break;
        tc_fence_after();
        // dV += P^T dO ; dK += dS^T Q     (M = keys, N = D, K = queries)
#pragma unroll
        for (int kk = 0; kk < kBM / 16; ++kk) {
          const uint32_t aoff = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          const uint32_t boff = kk * 2048;
          umma_f16_ss(tmem + C::kColDV, umma_desc_sw128(aP + aoff, 16, 1024),
                      umma_desc_sw128(aDO + boff, 128 * 128, 1024), id_acc, (t | kk) != 0);
          umma_f16_ss(tmem + C::kColDK, umma_desc_sw128(aDS + aoff, 16, 1024),
                      umma_desc_sw128(aQ + boff, 128 * 128, 1024), id_acc, (t | kk) != 0);
        }
        // dQ = dS K   (M = queries (dS^T read MN-major), N = D, K = keys)
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint32_t off = kk * 2048;
          umma_f16_ss(tmem + C::kColDQ, umma_desc_sw128(aDS + off, 128 * 128, 1024),
                      umma_desc_sw128(aK + off, 128 * 128, 1024), id_dq, kk > 0);
        }
        umma_commit(mm_done);
        umma_commit(&qdo_empty[st]);
      }
    }
  } else if (warp == pull_warp<SH>()) {
    pull_slice(p.pull, threadIdx.x & 31, 32);
  } else {
    // ---------------------------------------------------------------- softmax / dQ / epilogue
    static_assert(SH == 1 || SH == 2, "one or two softmax warp groups");
    const int quarter = warp & 3;
    const int half = SH == 1 ? 0 : (warp - 2) >> 2;   // softmax warp group: 0 .. SH-1
    const int lane = threadIdx.x & 31;
    const int row = quarter * 32 + lane;  // TMEM lane: key row (S^T, dP^T, dV, dK) / query row (dQ)
    const uint32_t lo = static_cast<uint32_t>(quarter * 32) << 16;
    const int krow = n0 + row;
    const int kpos = p.k_offset + krow;
    bool ok = true;
    // lse / delta of a step's query block: the first group's 128 threads read one value
    // each, one step ahead (issued before this step's dQ drain, so the global latency is
    // off the critical path), and publish them in shared memory at the step's start
    float lse_next = INFINITY, delta_next = 0.f;
    auto fetch_ld = [&](int t) {
      if (half != 0 || t >= total_steps) return;
      const int h = kvh * group + t / steps_per_head;
      const int q = (m_begin + t % steps_per_head) * kBM + row;
      const int64_t base = (static_cast<int64_t>(b) * p.Hq + h) * p.Sq;
      lse_next = q < p.Sq ? __ldg(p.lse + base + q) : INFINITY;
      delta_next = q < p.Sq ? __ldg(p.delta + base + q) : 0.f;
    };
    fetch_ld(0);
    for (int t = 0; t < total_steps; ++t) {
      const int h = kvh * group + t / steps_per_head;
      const int m0 = (m_begin + t % steps_per_head) * kBM;
      if (half == 0) {
        sLse[row] = lse_next;
        sDelta[row] = delta_next;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(128 * SH) : "memory");
      const bool tr = threadIdx.x == 64 && t < kTraceSteps;
      if (tr) trace_stamp(p, 3 + 6 * t);
      if (ok) ok = mbar_wait(sdp_full, t & 1, p.status, kStatusAttnTimeout, abort_flag);
      if (tr) trace_stamp(p, 3 + 6 * t + 1);
      ok = __all_sync(0xffffffffu, ok);  // keep TMEM ops warp-uniform
      if (!ok) continue;  // keep joining the named barrier until the loop ends
      tc_fence_after();
      // previous step's MMAs must be done with the P^T / dS^T tiles
      if (t > 0) {
        ok = mbar_wait(mm_done, (t - 1) & 1, p.status, kStatusAttnTimeout, abort_flag);
        ok = __all_sync(0xffffffffu, ok);  // keep TMEM ops warp-uniform
      if (!ok) continue;  // keep joining the named barrier until the loop ends
      }
      if (tr) trace_stamp(p, 3 + 6 * t + 2);
      const bool diag = p.causal && (p.k_offset + n0 + kBN - 1 > p.q_offset + m0);
      const bool tail = (m0 + kBM > p.Sq) || (n0 + kBN > p.Sk);
      // One 32-query chunk at a time: exponentiate, form dS, and store both bf16 chunks
      // straight into the swizzled P^T / dS^T tiles (keeps register pressure low). Each
      // softmax group takes its share of the chunks.
      constexpr int kChunks = kBM / 32 / SH;
#pragma unroll 1
      for (int c = half * kChunks; c < (half + 1) * kChunks; ++c) {
        uint32_t sr[32], dr[32];
        tmem_ld_32x32b_x32(tmem + lo + C::kColS + c * 32, sr);
        tmem_ld_32x32b_x32(tmem + lo + C::kColDP + c * 32, dr);
        // The chunk's 32 query statistics (the same for every thread), read as 16-byte
        // shared loads while the TMEM loads are in flight: one load latency per chunk
        // instead of one per element (per-element reads of these values, interleaved
        // with the tile stores, serialised the phase on load latency).
        float lq[32], dl[32];
        {
          const float4* l4 = reinterpret_cast<const float4*>(sLse + c * 32);
          const float4* d4 = reinterpret_cast<const float4*>(sDelta + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 a = l4[i], bq = d4[i];
            lq[4 * i] = a.x;
            lq[4 * i + 1] = a.y;
            lq[4 * i + 2] = a.z;
            lq[4 * i + 3] = a.w;
            dl[4 * i] = bq.x;
            dl[4 * i + 1] = bq.y;
            dl[4 * i + 2] = bq.z;
            dl[4 * i + 3] = bq.w;
          }
        }
        tmem_wait_ld();
        const bool trc = tr && t == 0 && c == half * kChunks;
        if (trc) trace_stamp(p, kTraceChunk);
        uint32_t ppk[16], dpk[16];
        // Visible query columns of this key row within the chunk: [vis_lo, vis_hi)
        // (all 32 outside diagonal / tail blocks); masked entries get P = 0 by a select.
        int vis_lo = 0, vis_hi = 32;
        if (diag || tail) {
          const int q0 = m0 + c * 32;
          vis_hi = krow < p.Sk ? min(32, p.Sq - q0) : 0;
          if (p.causal) vis_lo = max(0, kpos - p.q_offset - q0);
        }
        // Stage by stage over the 32 elements (all exponent arguments, then all
        // exponentials, then dS), so the 32 independent MUFU operations are in flight
        // together instead of one dependency chain per element.
        float pr[32], ds[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) pr[e] = fmaf(__uint_as_float(sr[e]), p.scale_log2, -lq[e]);
#pragma unroll
        for (int e = 0; e < 32; ++e) pr[e] = ex2(pr[e]);
#pragma unroll
        for (int e = 0; e < 32; ++e) pr[e] = (e >= vis_lo && e < vis_hi) ? pr[e] : 0.f;
#pragma unroll
        for (int e = 0; e < 32; ++e) ds[e] = pr[e] * (__uint_as_float(dr[e]) - dl[e]);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          ppk[e / 2] = pack_bf16x2(pr[e], pr[e + 1]);
          dpk[e / 2] = pack_bf16x2(ds[e], ds[e + 1]);
        }
        if (trc) trace_stamp(p, kTraceChunk + 1);
        store_chunk_sw128(sP, row, c, ppk);
        store_chunk_sw128(sDS, row, c, dpk);
        if (trc) trace_stamp(p, kTraceChunk + 2);
      }
      if (tr && t == 0) trace_stamp(p, kTraceChunk + 3);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pds_full);
      if (tr) trace_stamp(p, 3 + 6 * t + 3);
      fetch_ld(t + 1);
      // drain dQ (thread = query row m0 + row)
      ok = mbar_wait(mm_done, t & 1, p.status, kStatusAttnTimeout, abort_flag);
      ok = __all_sync(0xffffffffu, ok);  // keep TMEM ops warp-uniform
      if (!ok) continue;  // keep joining the named barrier until the loop ends
      if (tr) trace_stamp(p, 3 + 6 * t + 4);
      tc_fence_after();
      const int q = m0 + row;
      float* dst = p.dq_acc + ((static_cast<int64_t>(b) * p.Sq + q) * p.Hq + h) * D;
      constexpr int kDqChunks = D / 32 / SH;
#pragma unroll
      for (int c = half * kDqChunks; c < (half + 1) * kDqChunks; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + lo + C::kColDQ + c * 32, r);
        tmem_wait_ld();
        if (q < p.Sq) {
          if (p.dq_slot_stride != 0) {
            float4* sdst = reinterpret_cast<float4*>(dst + nb * p.dq_slot_stride + c * 32);
#pragma unroll
            for (int e = 0; e < 32; e += 4)
              sdst[e / 4] = make_float4(
                  __uint_as_float(r[e]) * p.scale, __uint_as_float(r[e + 1]) * p.scale,
                  __uint_as_float(r[e + 2]) * p.scale, __uint_as_float(r[e + 3]) * p.scale);
          } else {
#pragma unroll
            for (int e = 0; e < 32; e += 4)
              red_add_v4(dst + c * 32 + e, __uint_as_float(r[e]) * p.scale,
                         __uint_as_float(r[e + 1]) * p.scale, __uint_as_float(r[e + 2]) * p.scale,
                         __uint_as_float(r[e + 3]) * p.scale);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
      if (tr) trace_stamp(p, 3 + 6 * t + 5);
    }
    // ---- epilogue: dK (scaled, inverse RoPE) and dV for this thread's key row; with two
    // softmax groups the first writes dK and the second dV
    if (ok) {
      const bool have = total_steps > 0;
      if (have) tc_fence_after();
      // TMEM loads are warp-collective: every lane loads, only valid rows store.
      const bool row_ok = krow < p.Sk;
      const int krc = row_ok ? krow : 0;
      {
        __nv_bfloat16* dkr = p.dk + b * p.dk_batch + static_cast<int64_t>(krc) * p.dk_row +
                             static_cast<int64_t>(kvh) * D;
        __nv_bfloat16* dvr = p.dv + b * p.dv_batch + static_cast<int64_t>(krc) * p.dv_row +
                             static_cast<int64_t>(kvh) * D;
        const float pos = p.k_pos != nullptr ? static_cast<float>(__ldg(p.k_pos + krc)) : 0.f;
#pragma unroll
        for (int c = 0; c < (SH == 1 || half == 0 ? D / 64 : 0); ++c) {
          uint32_t a[32], bb[32];
          float x1[32], x2[32];
          if (have) {
            tmem_ld_32x32b_x32(tmem + lo + C::kColDK + c * 32, a);
            tmem_ld_32x32b_x32(tmem + lo + C::kColDK + D / 2 + c * 32, bb);
            tmem_wait_ld();
          }
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            x1[e] = have ? __uint_as_float(a[e]) * p.scale : 0.f;
            x2[e] = have ? __uint_as_float(bb[e]) * p.scale : 0.f;
          }
          if (p.k_cs != nullptr) {
            const float4* cs4 = reinterpret_cast<const float4*>(
                p.k_cs + static_cast<int64_t>(krc) * (D / 2) + c * 32);
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float4 t4 = __ldg(cs4 + e / 2);   // (cos_e, sin_e, cos_e+1, sin_e+1)
              float u = x1[e] * t4.x + x2[e] * t4.y;
              float w = x2[e] * t4.x - x1[e] * t4.y;
              x1[e] = u;
              x2[e] = w;
              u = x1[e + 1] * t4.z + x2[e + 1] * t4.w;
              w = x2[e + 1] * t4.z - x1[e + 1] * t4.w;
              x1[e + 1] = u;
              x2[e + 1] = w;
            }
          } else if (p.k_pos != nullptr) {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              float sn, cs;
              sincosf(pos * __ldg(p.inv_freq + c * 32 + e), &sn, &cs);
              const float u = x1[e] * cs + x2[e] * sn;
              const float w = x2[e] * cs - x1[e] * sn;
              x1[e] = u;
              x2[e] = w;
            }
          }
#pragma unroll
          for (int e = 0; e < 32 && row_ok; e += 8) {
            *reinterpret_cast<uint4*>(dkr + c * 32 + e) =
                make_uint4(pack_bf16x2(x1[e], x1[e + 1]), pack_bf16x2(x1[e + 2], x1[e + 3]),
                           pack_bf16x2(x1[e + 4], x1[e + 5]), pack_bf16x2(x1[e + 6], x1[e + 7]));
            *reinterpret_cast<uint4*>(dkr + D / 2 + c * 32 + e) =
                make_uint4(pack_bf16x2(x2[e], x2[e + 1]), pack_bf16x2(x2[e + 2], x2[e + 3]),
                           pack_bf16x2(x2[e + 4], x2[e + 5]), pack_bf16x2(x2[e + 6], x2[e + 7]));
          }
        }
#pragma unroll
        for (int c = 0; c < (SH == 1 || half == 1 ? D / 32 : 0); ++c) {
          uint32_t r[32];
          if (have) {
            tmem_ld_32x32b_x32(tmem + lo + C::kColDV + c * 32, r);
            tmem_wait_ld();
          }
#pragma unroll
          for (int e = 0; e < 32 && row_ok; e += 8) {
            float f[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) f[u] = have ? __uint_as_float(r[e + u]) : 0.f;
            *reinterpret_cast<uint4*>(dvr + c * 32 + e) =
                make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                           pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
          }
        }
      }
    }
  }
  if (threadIdx.x == 64) trace_stamp(p, 2);
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                                     cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && ptr != nullptr,
                "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

static CUtensorMap make_map(const at::Tensor& t) {
  CUtensorMap m;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(t.size(3)), static_cast<cuuint64_t>(t.size(2)),
                        static_cast<cuuint64_t>(t.size(1)), static_cast<cuuint64_t>(t.size(0))};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(t.stride(2) * 2),
                           static_cast<cuuint64_t>(t.stride(1) * 2),
                           static_cast<cuuint64_t>(t.stride(0) * 2)};
  cuuint32_t box[4] = {64u, 1u, 128u, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, t.data_ptr(), dims, strides,
                           box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "flash_attn_bwd_tc: tensor map encode failed (", (int)r, ")");
  return m;
}

}  // namespace fabw
}  // namespace nmb

using namespace nmb;
using namespace nmb::fabw;

PullDesc make_pull(int64_t src, const c10::optional<at::Tensor>& dst, int64_t flag, int64_t epoch,
                   int* status);   // attention_tc.cu

// Softmax warp groups per CTA: 2 (default; the P/dS phase is the longest of a step, and
// two groups halve it: +2.8 % on the 1-GPU 311M step) or 1 (NMB_ATTN_BWD_SOFTMAX_GROUPS=1).
static int softmax_groups() {
  static const int n = [] {
    const char* e = std::getenv("NMB_ATTN_BWD_SOFTMAX_GROUPS");
    return e != nullptr && std::atoi(e) == 1 ? 1 : 2;
  }();
  return n;
}

int64_t attn_bwd_softmax_groups() { return softmax_groups(); }

int64_t attn_bwd_trace_slots() { return kTraceSlots; }

template <int D, int SH>
static void launch_bwd(dim3 grid, cudaStream_t stream, const CUtensorMap& mq,
                       const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mdo,
                       const Params& p) {
  static bool set = false;
  if (!set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(flash_bwd_tc_kernel<D, SH>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        Cfg<D>::kSmem));
    set = true;
  }
  flash_bwd_tc_kernel<D, SH><<<grid, threads_for<SH>(), Cfg<D>::kSmem, stream>>>(mq, mk, mv,
                                                                                 mdo, p);
}

// dK / dV of the causal attention (tcgen05). `delta` (rowsum(dO*O)) and the
// zeroed fp32 `dq_acc` must be prepared by the caller (flash_attn_bwd_prep).
void flash_attn_bwd_tc_kv(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor dout,
                          at::Tensor lse, at::Tensor delta, at::Tensor dq_acc, at::Tensor dk,
                          at::Tensor dv, double softmax_scale, bool causal, int64_t q_offset,
                          int64_t k_offset, c10::optional<at::Tensor> k_pos,
                          c10::optional<at::Tensor> inv_freq, at::Tensor status,
                          int64_t pull_src, c10::optional<at::Tensor> pull_dst,
                          int64_t pull_flag, int64_t pull_epoch,
                          c10::optional<at::Tensor> k_cs, c10::optional<at::Tensor> trace,
                          int64_t dq_slot_stride) {
  const int64_t D = q.size(3);
  TORCH_CHECK(D == 64 || D == 128, "flash_attn_bwd_tc: head_dim must be 64 or 128");
  for (const at::Tensor* t : {&q, &k, &v, &dout, &dk, &dv}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 4);
    TORCH_CHECK(t->stride(3) == 1 && t->stride(2) == D, "heads must be contiguous [.., H, D]");
    TORCH_CHECK(t->stride(1) % 8 == 0 && t->stride(0) % 8 == 0, "strides must be 16-byte");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0, "16-byte alignment");
  }
  Params p{};
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  TORCH_CHECK(dq_acc.is_cuda() && dq_acc.scalar_type() == at::kFloat && dq_acc.is_contiguous() &&
                  (reinterpret_cast<uintptr_t>(dq_acc.data_ptr()) & 15u) == 0,
              "flash_attn_bwd_tc: dq_acc must be a contiguous, 16-byte aligned fp32 buffer");
  {
    const int64_t rows_d = q.size(0) * q.size(1) * q.size(2) * D;
    const int64_t slots = dq_slot_stride > 0 ? (k.size(1) + kBN - 1) / kBN : 1;
    TORCH_CHECK(dq_slot_stride == 0 || (dq_slot_stride >= rows_d && dq_slot_stride % 4 == 0),
                "flash_attn_bwd_tc: dq_slot_stride must be 0 or >= B*Sq*Hq*D and a multiple of 4");
    TORCH_CHECK(dq_acc.numel() >= (slots - 1) * dq_slot_stride + rows_d,
                "flash_attn_bwd_tc: dq_acc too small for ", slots, " slots");
  }
  p.dq_slot_stride = dq_slot_stride;
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.dk_row = dk.stride(1);
  p.dk_batch = dk.stride(0);
  p.dv_row = dv.stride(1);
  p.dv_batch = dv.stride(0);
  p.B = q.size(0);
  p.Sq = q.size(1);
  p.Hq = q.size(2);
  p.Sk = k.size(1);
  p.Hkv = k.size(2);
  p.q_offset = q_offset;
  p.k_offset = k_offset;
  p.causal = causal ? 1 : 0;
  p.scale = static_cast<float>(softmax_scale);
  p.scale_log2 = static_cast<float>(softmax_scale) * kLog2e;
  p.k_pos = k_pos.has_value() ? k_pos->data_ptr<int>() : nullptr;
  p.inv_freq = inv_freq.has_value() ? inv_freq->data_ptr<float>() : nullptr;
  TORCH_CHECK(p.k_pos == nullptr || p.inv_freq != nullptr);
  p.k_cs = nullptr;
  p.trace = nullptr;
  if (trace.has_value()) {
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong && trace->is_contiguous() &&
                    trace->numel() >= static_cast<int64_t>(k.size(2)) * q.size(0) *
                                          ((k.size(1) + kBN - 1) / kBN) * kTraceSlots,
                "flash_attn_bwd_tc: trace must be an int64 buffer of grid x ", kTraceSlots);
    p.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  if (k_cs.has_value() && p.k_pos != nullptr) {
    TORCH_CHECK(k_cs->is_cuda() && k_cs->scalar_type() == at::kFloat && k_cs->is_contiguous() &&
                    k_cs->numel() >= k.size(1) * D,
                "flash_attn_bwd_tc: k_cs must be a contiguous fp32 [Sk, D/2, 2] table");
    p.k_cs = reinterpret_cast<const float2*>(k_cs->data_ptr<float>());
  }
  p.status = status.data_ptr<int>();
  p.pull = make_pull(pull_src, pull_dst, pull_flag, pull_epoch, p.status);
  if (p.B == 0 || p.Sk == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  ensure_current_context(q.device().index());
  CUtensorMap mq = make_map(q), mk = make_map(k), mv = make_map(v), mdo = make_map(dout);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(static_cast<int64_t>(p.Hkv) * p.B < (1ll << 31) && (p.Sk + kBN - 1) / kBN < 65536);
  dim3 grid(p.Hkv * p.B, (p.Sk + kBN - 1) / kBN, 1);
  if (D == 64) {
    if (softmax_groups() == 2)
      launch_bwd<64, 2>(grid, stream, mq, mk, mv, mdo, p);
    else
      launch_bwd<64, 1>(grid, stream, mq, mk, mv, mdo, p);
  } else {
    if (softmax_groups() == 2)
      launch_bwd<128, 2>(grid, stream, mq, mk, mv, mdo, p);
    else
      launch_bwd<128, 1>(grid, stream, mq, mk, mv, mdo, p);
  }
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

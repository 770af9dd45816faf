// Persistent, warp-specialised bf16 GEMM for sm_100a on the 5th-generation
// tensor cores (tcgen05 + TMEM), operands staged by TMA.
//
//   C[m, n] = epilogue( sum_k A(m, k) * B(n, k) )
//
// A(m, k) is read from a [M, K] row-major tensor (K-major) or from a [K, M]
// tensor (MN-major); likewise B from [N, K] or [K, N]. All three products a
// transformer linear layer needs map onto this one kernel without transposes:
//   forward  y  = x W^T    A = x  (K-major), B = W  (K-major)
//   dgrad    dx = dy W     A = dy (K-major), B = W  (MN-major)
//   wgrad    dW = dy^T x   A = dy (MN-major), B = x (MN-major)
//
// Roles (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0   : TMA producer, one elected lane, ring of `kStages` smem stages
//   warp 1   : TMEM allocator + MMA issuer (one elected lane issues tcgen05.mma)
//   warps 2-5: epilogue; each thread owns one accumulator row (TMEM lane) and
//              drains it with tcgen05.ld, applies the fused epilogue, stores.
// The accumulator is double buffered in TMEM (2 x BN fp32 columns) so the
// epilogue of tile i overlaps the main loop of tile i+1.
//
// Fused epilogues:
//   kEpiBF16   : C(bf16) = alpha * acc (+ residual)
//   kEpiF32Acc : C(fp32) = beta * C + alpha * acc   (weight-gradient accumulation)
//   kEpiSwiGLU : B = [W_gate; W_up]; each BN tile carries BN/2 gate and BN/2 up
//                columns; writes h = silu(g) * u and keeps [g | u] for backward
//   kEpiRoPE   : rotate-half rotary embedding applied to the first `rope_cols`
//                columns (q and k heads) of a fused QKV projection
//   kEpiCEStats: LM head. Stores the bf16 logits and, per row, the (max, sum exp) of the
//                rounded logits over each epilogue warp's half of the tile into `ce_part`
//                ([M][n-tiles x 2] float2), so the cross-entropy needs no statistics pass
//                over the logits (it merges the parts, then writes the gradient in place)
//   kEpiPeer   : GEMM -> reduce-scatter. Output row r belongs to TP rank
//                r / comm_rows; the bf16 partial tile is stored straight into that
//                rank's symmetric staging buffer (slot = this rank) over NVLink, so
//                the transfer overlaps the remaining tiles. With the reduction in the
//                kernel (rs_inplace), the other ranks' rows are computed first, each of
//                their tiles followed by a per-tile flag in the owner's memory; this
//                rank's own rows come last, and their epilogue waits (bounded) for the
//                peers' tile flags and writes out = acc + the peers' partials + residual,
//                so the own partial never leaves the SM and no second pass runs. Without
//                it a flag-gated reduce kernel on the owner sums the slots (comm_ops.cu).
//
// Gathered A (template GATHER, AG -> GEMM): A's rows are split over the TP ranks,
// rank r's [comm_rows, K] shard living in r's symmetric buffer. The producer
// TMA-loads each tile from its owner's shard (a peer pointer mapped into this
// process; plain TMA, no multicast) after a bounded wait on the owner's "shard
// ready" flag. For n-tile 0 the MMA warp also TMA-stores the staged A tile into a
// local [M, K] buffer (materialising the gathered input the backward pass needs without
// a separate all-gather) and, once those stores are written, publishes a per-m-tile flag.
// Tiles are ordered so every remote row crosses NVLink once: first n-tile 0 of the
// peers' m-tiles, then all tiles of this rank's own rows, then the remaining n-tiles of
// the peers' rows, which read A from the local copy (a brief poll of the m-tile flag;
// a tile that finds it unset reads from the peer instead, so no new wait is introduced).
//
// The peer epilogue stages each 32 x 64 bf16 block of a warp in shared memory and writes
// it to the owner as 128-byte row segments (8 lanes per row), not as one 16-byte piece
// per row and lane: full-line writes over NVLink.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace nmb {

enum EpiKind : int {
  kEpiBF16 = 0, kEpiF32Acc = 1, kEpiSwiGLU = 2, kEpiRoPE = 3, kEpiPeer = 4, kEpiCEStats = 5
};
// LM head with cross-entropy statistics: each epilogue warp covers half of a 256-column tile
constexpr int kCEPartsPerTile = 2;

constexpr int kMaxTP = 8;
// Per-tile flags of the in-kernel GEMM -> reduce-scatter: every rank's buffer holds
// [TP senders][kRsTileFlags] epochs (a tile's index counts the owner's 128-row tiles x the
// N tiles), written by the sender after the tile's partial has been stored.
constexpr int kRsTileFlags = 16384;

struct GemmParams {
  int M, N, K;               // N = output columns (for SwiGLU: F, the gate/up width)
  void* C;                   // output
  int64_t ldc;               // output row pitch, elements
  const __nv_bfloat16* R;    // optional bf16 residual added in kEpiBF16
  int64_t ldr;
  const float* alpha_ptr;    // optional device scalar multiplying the accumulator
  float alpha;
  float beta;                // kEpiF32Acc: 0 overwrites, 1 accumulates
  __nv_bfloat16* aux;        // kEpiSwiGLU: [M, 2F] store of gate | up
  int64_t ld_aux;
  int swiglu_up_row;         // kEpiSwiGLU: row of W_up inside B (= F)
  const int* positions;      // kEpiRoPE: position of each sequence slot [seq_len]
  int seq_len;
  int pos_div;               // kEpiRoPE: row r has position positions[(r / pos_div) % seq_len]
  const float* inv_freq;     // kEpiRoPE: [head_dim / 2]
  int head_dim;
  int rope_cols;
  int* status;
  int num_m_tiles, num_n_tiles;
  // Tensor-parallel communication (gathered A / peer epilogue).
  int comm_rows;                        // rows of A (gather) or C (peer) owned per TP rank
  int comm_rank, comm_size;
  const uint32_t* flags;                // gather: this rank's flags, slot r = rank r's epoch
  const uint32_t* epoch_ptr;            // device epoch counter of the collective's channel
  int m_rotate;                         // gather: first M tile (own rows first)
  int store_gathered;                   // gather: TMA-store A tiles into `xfull`
  __nv_bfloat16* peer_out[2][kMaxTP];   // peer epilogue: [parity][rank] staging bases
  int splits;                           // split-K factor (kEpiF32Acc with beta = 1 only)
  const float2* rope_cs;                // kEpiRoPE: (cos, sin) table [seq_len][head_dim / 2]
  const uint32_t* rope_cs16;            // kEpiRoPE: the same table as packed bf16 (cos | sin)
  uint32_t* gather_ready;               // gather: per m-tile "rows staged in xfull" = epoch
  float2* ce_part;                      // kEpiCEStats: [M][num_n_tiles * kCEPartsPerTile]
  // GEMM -> reduce-scatter with the reduction in the epilogue (kEpiPeer, rs_inplace = 1)
  uint32_t* tile_flags[kMaxTP];         // per owner rank: its [TP][kRsTileFlags] flag array
  __nv_bfloat16* own_out;               // this rank's reduced rows [comm_rows, N]
  int64_t ld_own;
  int rs_inplace;
};

// Per-rank tensor maps of the gathered A operand and of the local gathered copy.
// The epoch lives in device memory (advanced by the signal kernel), so a launch carries
// no per-call value and the whole sequence can be captured in a CUDA graph; the data
// buffers alternate by epoch parity, hence two sets of shard maps / staging pointers.
struct CommMaps {
  CUtensorMap a[2][kMaxTP];
  CUtensorMap xfull;
};

constexpr int kBM = 128;
constexpr int kBK = 64;                // one 128-byte swizzle row of bf16
// Epilogue warps: two per TMEM lane quarter (each drains half of the tile's columns), so
// two warps per SM sub-partition overlap their TMEM loads, global loads and math.
template <int EPI>
__host__ __device__ constexpr int epi_warps() { return 8; }
template <int EPI>
__host__ __device__ constexpr int gemm_threads() { return 64 + 32 * epi_warps<EPI>(); }
constexpr int kUmmaK = 16;

template <int BN, int EPI>
struct GemmCfg {
  // the peer epilogue's per-warp staging area (36 KB) takes one stage
  static constexpr int kStages = (BN == 256 ? 4 : 6) - (EPI == kEpiPeer ? 1 : 0);
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;  // double-buffered accumulator
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// Peer epilogue staging: per epilogue warp 32 rows x 64 bf16 (+16 B pad per row, so the
// row-wise writes and the segment-wise reads are both free of bank conflicts).
constexpr int kPeerRowBytes = 64 * 2 + 16;
constexpr int kPeerStageBytes = 8 * 32 * kPeerRowBytes;
// How long a gather tile polls for the local copy of its rows before reading the peer.
constexpr unsigned long long kLocalCopyPollNs = 20000ull;

template <int BN, int EPI>
constexpr int gemm_smem_bytes() {
  return GemmCfg<BN, EPI>::kSmemBytes + (EPI == kEpiPeer ? kPeerStageBytes : 0);
}

// silu(x) = x / (1 + e^-x) with the fast reciprocal-based division (the result is
// rounded to bf16); for x < -87, e^-x is +inf and the quotient is -0, the limit.
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// v[0..8) += the 8 bf16 values of a 16-byte word.
__device__ __forceinline__ void add_bf16x8(float* v, const uint4 w) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    v[2 * e] += bf16_lo(u[e]);
    v[2 * e + 1] += bf16_hi(u[e]);
  }
}

// Store 32 fp32 values as bf16 to row pointer `dst` (cols [col, col+32)), predicated on N.
__device__ __forceinline__ void store_row32_bf16(__nv_bfloat16* dst, int col, int ncols,
                                                 const float (&v)[32]) {
  if (col + 32 <= ncols && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w;
      w.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
      w.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
      w.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
      w.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
      d4[q] = w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col + j < ncols) dst[j] = __float2bfloat16_rn(v[j]);
  }
}

// Work item t -> output tile (m0, nt) and K-split ks. Splits are the slowest index so the
// concurrently running CTAs of one split share A/B panels in L2.
template <bool GATHER>
__device__ __forceinline__ void tile_coords(int t, const GemmParams& p, int& m0, int& nt,
                                            int& ks) {
  if constexpr (GATHER) {
    // remote m-tiles x n-tile 0 | own m-tiles x all n-tiles | remote m-tiles x n-tiles >= 1
    const int own = p.comm_rows / kBM;
    const int rem = p.num_m_tiles - own;
    const int own0 = p.comm_rank * own;
    ks = 0;
    if (t < rem) {
      m0 = ((own0 + own + t) % p.num_m_tiles) * kBM;
      nt = 0;
      return;
    }
    t -= rem;
    if (t < own * p.num_n_tiles) {
      m0 = (own0 + t % own) * kBM;
      nt = t / own;
      return;
    }
    t -= own * p.num_n_tiles;
    m0 = ((own0 + own + t % rem) % p.num_m_tiles) * kBM;
    nt = 1 + t / rem;
    return;
  }
  const int per_split = p.num_m_tiles * p.num_n_tiles;
  ks = t / per_split;
  t -= ks * per_split;
  const int mt = t % p.num_m_tiles;
  m0 = mt * kBM;
  nt = t / p.num_m_tiles;
}

// Work item t -> tile, per epilogue kind. The in-kernel GEMM -> reduce-scatter orders the
// other ranks' rows first (their partials travel while this rank computes the rest) and
// this rank's own rows last (their epilogue waits for the peers' partials).
template <int EPI, bool GATHER>
__device__ __forceinline__ void work_coords(int t, const GemmParams& p, int& m0, int& nt,
                                            int& ks) {
  if constexpr (EPI == kEpiPeer) {
    if (p.rs_inplace) {
      const int own = p.comm_rows / kBM, rem = p.num_m_tiles - own, own0 = p.comm_rank * own;
      ks = 0;
      if (t < rem * p.num_n_tiles) {
        m0 = ((own0 + own + t % rem) % p.num_m_tiles) * kBM;
        nt = t / rem;
        return;
      }
      t -= rem * p.num_n_tiles;
      m0 = (own0 + t % own) * kBM;
      nt = t / own;
      return;
    }
  }
  tile_coords<GATHER>(t, p, m0, nt, ks);
}

// Brief, bounded poll of a gather m-tile's local-copy flag; false = not there (yet).
__device__ __forceinline__ bool poll_local_copy(const uint32_t* flag, uint32_t epoch) {
  if (ld_acquire_gpu(flag) == epoch) return true;
  const unsigned long long start = globaltimer_ns();
  for (uint32_t it = 0; it < 4096u; ++it) {
    __nanosleep(32);
    if (ld_acquire_gpu(flag) == epoch) return true;
    if (globaltimer_ns() - start > kLocalCopyPollNs) break;
  }
  return false;
}

__device__ __forceinline__ void split_range(const GemmParams& p, int num_kb, int ks, int& kb0,
                                            int& kb1) {
  const int per = (num_kb + p.splits - 1) / p.splits;
  kb0 = ks * per;
  kb1 = min(num_kb, kb0 + per);
}

// Vectorised fp32 atomic add (sm_90+): out[0..3] += v (16-byte aligned).
__device__ __forceinline__ void red_add_v4(float* out, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(out), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool GATHER>
__global__ void __launch_bounds__(gemm_threads<EPI>(), 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CommMaps cm, const GemmParams p) {
  using Cfg = GemmCfg<BN, EPI>;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + S * Cfg::kABytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* tfull_bar = empty_bar + S;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* peer_stage = smem + S * Cfg::kStageBytes + 256;   // kEpiPeer only

  const int warp = threadIdx.x / 32;
  const int num_tiles = p.num_m_tiles * p.num_n_tiles * p.splits;
  const int num_kb = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], epi_warps<EPI>());  // one arrive per epilogue warp
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t ready = GATHER ? (1u << p.comm_rank) : 0u;
      uint32_t epoch = 0;
      if constexpr (GATHER) epoch = *reinterpret_cast<const volatile uint32_t*>(p.epoch_ptr);
      const int par = static_cast<int>(epoch & 1u);
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int m0, nt, ks, kb0, kb1;
        work_coords<EPI, GATHER>(t, p, m0, nt, ks);
        split_range(p, num_kb, ks, kb0, kb1);
        int owner = 0;
        bool from_local = false;
        if constexpr (GATHER) {
          owner = m0 / p.comm_rows;
          if (owner != p.comm_rank && nt > 0 && p.store_gathered && p.gather_ready != nullptr) {
            from_local = poll_local_copy(p.gather_ready + m0 / kBM, epoch);
            if (from_local) fence_proxy_async_global();
          }
          if (!from_local && !((ready >> owner) & 1u)) {
            if (!wait_flag(p.flags + owner, epoch, p.status, kStatusPeerFlagTimeout,
                           abort_flag)) {
              ok = false;
              break;
            }
            fence_proxy_async_global();
            ready |= 1u << owner;
          }
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, p.status, kStatusGemmProducerTimeout,
                         abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageBytes);
          uint8_t* sa = smem_a + stage * Cfg::kABytes;
          uint8_t* sb = smem_b + stage * Cfg::kBBytes;
          const int k0 = kb * kBK;
          if constexpr (GATHER) {
            if (from_local)
              tma_load_2d(sa, &cm.xfull, &full_bar[stage], k0, m0);
            else
              tma_load_2d(sa, &cm.a[par][owner], &full_bar[stage], k0, m0 - owner * p.comm_rows);
          } else if constexpr (!A_MN) {
            tma_load_2d(sa, &tmA, &full_bar[stage], k0, m0);
          } else {
            tma_load_2d(sa, &tmA, &full_bar[stage], m0, k0);
            tma_load_2d(sa + kBK * 128, &tmA, &full_bar[stage], m0 + 64, k0);
          }
          if constexpr (EPI == kEpiSwiGLU) {
            const int n0h = nt * (BN / 2);
            tma_load_2d(sb, &tmB, &full_bar[stage], k0, n0h);
            tma_load_2d(sb + (BN / 2) * 128, &tmB, &full_bar[stage], k0, p.swiglu_up_row + n0h);
          } else if constexpr (!B_MN) {
            tma_load_2d(sb, &tmB, &full_bar[stage], k0, nt * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sb + j * kBK * 128, &tmB, &full_bar[stage], nt * BN + j * 64, k0);
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      uint32_t gepoch = 0;
      if constexpr (GATHER) gepoch = *reinterpret_cast<const volatile uint32_t*>(p.epoch_ptr);
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, p.status, kStatusGemmMmaTimeout,
                       abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        int m0 = 0, nt = 0, ks = 0, kb0 = 0, kb1 = 0;
        work_coords<EPI, GATHER>(t, p, m0, nt, ks);
        split_range(p, num_kb, ks, kb0, kb1);
        const bool store_a = GATHER && p.store_gathered && nt == 0;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, p.status, kStatusGemmMmaTimeout, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (store_a) {
            tma_store_2d(&cm.xfull, smem_a + stage * Cfg::kABytes, kb * kBK, m0);
            tma_store_commit();
          }
          const uint32_t a_addr = smem_u32(smem_a + stage * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(smem_b + stage * Cfg::kBBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
            uint64_t adesc, bdesc;
            if constexpr (!A_MN)
              adesc = umma_desc_sw128(a_addr + kk * 32, 16, 1024);
            else
              adesc = umma_desc_sw128(a_addr + kk * 2048, kBK * 128, 1024);
            if constexpr (!B_MN)
              bdesc = umma_desc_sw128(b_addr + kk * 32, 16, 1024);
            else
              bdesc = umma_desc_sw128(b_addr + kk * 2048, kBK * 128, 1024);
            umma_f16_ss(tmem_d, adesc, bdesc, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
          }
          if (store_a) tma_store_wait_read();  // the stage is refilled once released
          umma_commit(&empty_bar[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);
        if (store_a && p.gather_ready != nullptr) {
          // the tile's rows are in xfull once the bulk stores are written: publish them
          tma_store_wait_all();
          fence_proxy_async_global();
          st_release_gpu(p.gather_ready + m0 / kBM, gepoch);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    // column share of this warp: part `ew` of `kParts` equal parts of the tile
    constexpr int kParts = epi_warps<EPI>() / 4;
    const int ew = (warp - 2) / 4;
    const int lane = threadIdx.x & 31;
    const float alpha = p.alpha_ptr != nullptr ? p.alpha * __ldg(p.alpha_ptr) : p.alpha;
    // peer epilogue: this call's epoch is the next one (the signal kernel advances it later)
    int out_par = 0;
    uint32_t out_epoch = 0;
    if constexpr (EPI == kEpiPeer) {
      out_epoch = *reinterpret_cast<const volatile uint32_t*>(p.epoch_ptr) + 1u;
      out_par = static_cast<int>(out_epoch & 1u);
    }
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, p.status, kStatusGemmEpilogueTimeout,
                     abort_flag))
        break;
      tc_fence_after();
      int m0, nt, ks;
      work_coords<EPI, GATHER>(t, p, m0, nt, ks);
      const int row = m0 + quarter * 32 + lane;
      const bool row_ok = row < p.M;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;

      if constexpr (EPI == kEpiPeer) {
        // every row of a 128-row tile has the same owner (rows per rank % 128 == 0)
        const int owner = m0 / p.comm_rows;
        const int n0 = nt * BN;
        const int tile_local = ((m0 - owner * p.comm_rows) / kBM) * p.num_n_tiles + nt;
        if (p.rs_inplace && owner == p.comm_rank) {
          // own rows: every peer's partial of this tile must have landed (bounded wait on
          // the per-tile flags it wrote after its stores), then out = acc + partials (+ res)
          bool landed = true;
          for (int src = 0; src < p.comm_size && landed; ++src)
            if (src != p.comm_rank)
              landed = wait_flag(p.tile_flags[p.comm_rank] + src * kRsTileFlags + tile_local,
                                 out_epoch, p.status, kStatusPeerFlagTimeout, abort_flag);
          if (landed) {
            const int lrow = row - p.comm_rank * p.comm_rows;
            const __nv_bfloat16* stg = p.peer_out[out_par][p.comm_rank];  // [TP][rows][ldc]
            constexpr int kChunks = BN / 32 / kParts;
#pragma unroll 1
            for (int c = ew * kChunks; c < (ew + 1) * kChunks; ++c) {
              const int col = n0 + c * 32;
              uint32_t r[32];
              tmem_ld_32x32b_x32(tbase + c * 32, r);
              float v[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = 0.f;
              const bool vec = col + 32 <= p.N;
              // the residual and the peers' partials load while the TMEM load is in flight
              if (vec) {
                if (p.R != nullptr) {
                  const uint4* rr = reinterpret_cast<const uint4*>(
                      p.R + static_cast<int64_t>(lrow) * p.ldr + col);
#pragma unroll
                  for (int q = 0; q < 4; ++q) add_bf16x8(v + 8 * q, __ldg(rr + q));
                }
                for (int src = 0; src < p.comm_size; ++src) {
                  if (src == p.comm_rank) continue;
                  const uint4* sp = reinterpret_cast<const uint4*>(
                      stg + (static_cast<int64_t>(src) * p.comm_rows + lrow) * p.ldc + col);
#pragma unroll
                  for (int q = 0; q < 4; ++q) add_bf16x8(v + 8 * q, __ldcg(sp + q));
                }
              }
              tmem_wait_ld();
              if (col >= p.N) continue;
              __nv_bfloat16* orow = p.own_out + static_cast<int64_t>(lrow) * p.ld_own;
              if (vec) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += __uint_as_float(r[j]) * alpha;
                store_row32_bf16(orow + col, col, p.N, v);
              } else {
                for (int j = 0; j < 32 && col + j < p.N; ++j) {
                  float x = __uint_as_float(r[j]) * alpha;
                  if (p.R != nullptr)
                    x += __bfloat162float(p.R[static_cast<int64_t>(lrow) * p.ldr + col + j]);
                  for (int src = 0; src < p.comm_size; ++src)
                    if (src != p.comm_rank)
                      x += __bfloat162float(
                          stg[(static_cast<int64_t>(src) * p.comm_rows + lrow) * p.ldc + col + j]);
                  orow[col + j] = __float2bfloat16_rn(x);
                }
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty_bar[acc]);
          continue;
        }
        __nv_bfloat16* base = p.peer_out[out_par][owner] +
                              static_cast<int64_t>(p.comm_rank * p.comm_rows - owner * p.comm_rows) *
                                  p.ldc;
        uint8_t* wst = peer_stage + (warp - 2) * 32 * kPeerRowBytes;
        constexpr int kC2 = BN / 64 / kParts;   // 64-column blocks of this warp
#pragma unroll 1
        for (int c2 = ew * kC2; c2 < (ew + 1) * kC2; ++c2) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tbase + (2 * c2 + h) * 32, r);
            tmem_wait_ld();
            uint4* d = reinterpret_cast<uint4*>(wst + lane * kPeerRowBytes + h * 64);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(r[8 * q + 0]) * alpha,
                                __uint_as_float(r[8 * q + 1]) * alpha);
              w.y = pack_bf16x2(__uint_as_float(r[8 * q + 2]) * alpha,
                                __uint_as_float(r[8 * q + 3]) * alpha);
              w.z = pack_bf16x2(__uint_as_float(r[8 * q + 4]) * alpha,
                                __uint_as_float(r[8 * q + 5]) * alpha);
              w.w = pack_bf16x2(__uint_as_float(r[8 * q + 6]) * alpha,
                                __uint_as_float(r[8 * q + 7]) * alpha);
              d[q] = w;
            }
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int rr = i * 4 + (lane >> 3);
            const int grow = m0 + quarter * 32 + rr;
            const int gcol = n0 + c2 * 64 + (lane & 7) * 8;
            if (grow < p.M && gcol < p.N) {
              const uint4 v = *reinterpret_cast<const uint4*>(wst + rr * kPeerRowBytes +
                                                              (lane & 7) * 16);
              *reinterpret_cast<uint4*>(base + static_cast<int64_t>(grow) * p.ldc + gcol) = v;
            }
          }
          __syncwarp();
        }
        if (p.rs_inplace) {
          // the owner may read this tile once every epilogue warp's stores are visible
          asm volatile("bar.sync 2, %0;" ::"n"(32 * epi_warps<EPI>()) : "memory");
          if (threadIdx.x == 64)   // release at system scope: cumulative over the barrier
            st_release_sys(p.tile_flags[owner] + p.comm_rank * kRsTileFlags + tile_local,
                           out_epoch);
        }
      } else if constexpr (EPI == kEpiBF16 || EPI == kEpiF32Acc) {
        const int n0 = nt * BN;
        constexpr int kChunks = BN / 32 / kParts;   // 32-column chunks of this warp
        const int c_begin = ew * kChunks, c_end = c_begin + kChunks;
        // Residual (kEpiBF16): each thread reads its own row, 32 columns = 64 bytes per
        // chunk, as four 16-byte loads issued one chunk ahead of their use, so the global
        // latency overlaps the TMEM drain of the previous chunk.
        const bool res_vec = EPI == kEpiBF16 && p.R != nullptr && row_ok &&
                             (p.ldr % 8) == 0 && (reinterpret_cast<uintptr_t>(p.R) & 15u) == 0;
        const uint4* res_row =
            res_vec ? reinterpret_cast<const uint4*>(p.R + static_cast<int64_t>(row) * p.ldr + n0)
                    : nullptr;
        uint4 res_next[4];
        if (res_vec && n0 + (c_begin + 1) * 32 <= p.N) {
#pragma unroll
          for (int q = 0; q < 4; ++q) res_next[q] = __ldg(res_row + c_begin * 4 + q);
        }
#pragma unroll 1
        for (int c = c_begin; c < c_end; ++c) {
          uint4 res_cur[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) res_cur[q] = res_next[q];
          if (res_vec && c + 1 < c_end && n0 + (c + 2) * 32 <= p.N) {
#pragma unroll
            for (int q = 0; q < 4; ++q) res_next[q] = __ldg(res_row + (c + 1) * 4 + q);
          }
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c * 32, r);
          tmem_wait_ld();
          const int col = n0 + c * 32;
          if (!row_ok || col >= p.N) continue;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * alpha;
          if constexpr (EPI == kEpiBF16) {
            if (res_vec && col + 32 <= p.N) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint32_t w[4] = {res_cur[q].x, res_cur[q].y, res_cur[q].z, res_cur[q].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  v[q * 8 + 2 * e] += bf16_lo(w[e]);
                  v[q * 8 + 2 * e + 1] += bf16_hi(w[e]);
                }
              }
            } else if (p.R != nullptr) {
              const __nv_bfloat16* rr = p.R + static_cast<int64_t>(row) * p.ldr + col;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col + j < p.N) v[j] += __bfloat162float(rr[j]);
            }
            store_row32_bf16(reinterpret_cast<__nv_bfloat16*>(p.C) +
                                 static_cast<int64_t>(row) * p.ldc + col,
                             col, p.N, v);
          } else {
            float* cp = reinterpret_cast<float*>(p.C) + static_cast<int64_t>(row) * p.ldc + col;
            if (p.splits > 1) {  // split-K partial sums: accumulate in L2 with atomics
              if (col + 32 <= p.N && (reinterpret_cast<uintptr_t>(cp) & 15u) == 0) {
#pragma unroll
                for (int q = 0; q < 8; ++q)
                  red_add_v4(cp + 4 * q, v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
              } else {
                for (int j = 0; j < 32; ++j)
                  if (col + j < p.N) atomicAdd(cp + j, v[j]);
              }
            } else if (col + 32 <= p.N) {
              float4* c4 = reinterpret_cast<float4*>(cp);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                float4 o = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                if (p.beta != 0.0f) {
                  const float4 old = c4[q];
                  o.x += p.beta * old.x;
                  o.y += p.beta * old.y;
                  o.z += p.beta * old.z;
                  o.w += p.beta * old.w;
                }
                c4[q] = o;
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (col + j < p.N) cp[j] = v[j] + (p.beta != 0.0f ? p.beta * cp[j] : 0.0f);
            }
          }
        }
      } else if constexpr (EPI == kEpiSwiGLU) {
        const int n0h = nt * (BN / 2);
        constexpr int kChunks = BN / 64 / kParts;   // 32-column gate/up chunk pairs
#pragma unroll 1
        for (int c = ew * kChunks; c < (ew + 1) * kChunks; ++c) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(tbase + c * 32, g);
          tmem_ld_32x32b_x32(tbase + BN / 2 + c * 32, u);
          tmem_wait_ld();
          const int col = n0h + c * 32;
          if (!row_ok || col >= p.N) continue;
          float gv[32], uv[32], hv[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            gv[j] = __uint_as_float(g[j]);
            uv[j] = __uint_as_float(u[j]);
            // Round through bf16 so forward and backward see the same g, u.
            gv[j] = __bfloat162float(__float2bfloat16_rn(gv[j]));
            uv[j] = __bfloat162float(__float2bfloat16_rn(uv[j]));
            hv[j] = silu_f(gv[j]) * uv[j];
          }
          store_row32_bf16(reinterpret_cast<__nv_bfloat16*>(p.C) +
                               static_cast<int64_t>(row) * p.ldc + col,
                           col, p.N, hv);
          __nv_bfloat16* arow = p.aux + static_cast<int64_t>(row) * p.ld_aux;
          store_row32_bf16(arow + col, col, p.N, gv);
          store_row32_bf16(arow + p.N + col, col, p.N, uv);
        }
      } else if constexpr (EPI == kEpiCEStats) {
        static_assert(kParts == kCEPartsPerTile, "one statistics part per epilogue warp half");
        const int n0 = nt * BN;
        constexpr int kChunks = BN / 32 / kParts;
        constexpr float kLog2e = 1.4426950408889634f;
        float m = -INFINITY, sx = 0.f;
        __nv_bfloat16* crow =
            reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(row) * p.ldc;
#pragma unroll 1
        for (int c = ew * kChunks; c < (ew + 1) * kChunks; ++c) {
          const int col = n0 + c * 32;
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c * 32, r);
          tmem_wait_ld();
          if (!row_ok || col >= p.N) continue;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j)   // the values the cross-entropy will read back
            v[j] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[j]) * alpha));
          store_row32_bf16(crow + col, col, p.N, v);
          const int nv = min(32, p.N - col);
          float lm = -INFINITY;
#pragma unroll
          for (int j = 0; j < 32; ++j) lm = j < nv ? fmaxf(lm, v[j]) : lm;
          const float nm = fmaxf(m, lm);
          float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int j = 0; j < 32; ++j)
            part[j & 3] += j < nv ? ex2_approx((v[j] - nm) * kLog2e) : 0.f;
          sx = (m == -INFINITY ? 0.f : sx * ex2_approx((m - nm) * kLog2e)) +
               ((part[0] + part[1]) + (part[2] + part[3]));
          m = nm;
        }
        if (row_ok)
          p.ce_part[(static_cast<int64_t>(row) * p.num_n_tiles + nt) * kCEPartsPerTile + ew] =
              make_float2(m, sx);
      } else {  // kEpiRoPE
        const int n0 = nt * BN;
        const int D = p.head_dim;
        const int half_chunks = D / 64;  // 32-col chunks per half head
        const int chunks_per_head = D / 32;
        const int slot = row_ok ? (row / p.pos_div) % p.seq_len : 0;
        const int pos = row_ok ? __ldg(p.positions + slot) : 0;
        // (head, half-chunk) pairs of the tile, dealt round-robin to the kParts warps
        const int pairs = (BN / D) * half_chunks;
        // bf16 (cos, sin) of this row's position for the current half-chunk, loaded once
        // and reused by every head of the tile that rotates with the same frequencies
        uint32_t cs16[32];
        int cs16_j = -1;
#pragma unroll 1
        for (int i = ew; i < pairs; i += kParts) {
          {
            const int h = i / half_chunks, j = i % half_chunks;
            const int c_lo = h * chunks_per_head + j;
            const int c_hi = c_lo + half_chunks;
            uint32_t lo[32], hi[32];
            tmem_ld_32x32b_x32(tbase + c_lo * 32, lo);
            tmem_ld_32x32b_x32(tbase + c_hi * 32, hi);
            tmem_wait_ld();
            const int col_lo = n0 + c_lo * 32;
            const int col_hi = n0 + c_hi * 32;
            if (!row_ok || col_lo >= p.N) continue;
            float a[32], b[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              a[e] = __uint_as_float(lo[e]) * alpha;
              b[e] = __uint_as_float(hi[e]) * alpha;
            }
            if (col_lo < p.rope_cols) {
              if (p.rope_cs16 != nullptr) {
                if (j != cs16_j) {
                  const uint4* t4 = reinterpret_cast<const uint4*>(
                      p.rope_cs16 + static_cast<int64_t>(slot) * (D / 2) + j * 32);
#pragma unroll
                  for (int q = 0; q < 8; ++q) {
                    const uint4 w = __ldg(t4 + q);
                    cs16[4 * q] = w.x;
                    cs16[4 * q + 1] = w.y;
                    cs16[4 * q + 2] = w.z;
                    cs16[4 * q + 3] = w.w;
                  }
                  cs16_j = j;
                }
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                  const float cs = bf16_lo(cs16[e]), sn = bf16_hi(cs16[e]);
                  const float x1 = a[e], x2 = b[e];
                  a[e] = x1 * cs - x2 * sn;
                  b[e] = x2 * cs + x1 * sn;
                }
              } else if (p.rope_cs != nullptr) {  // precomputed (cos, sin) of this row's slot
                const float4* cs4 = reinterpret_cast<const float4*>(
                    p.rope_cs + static_cast<int64_t>(slot) * (D / 2) + j * 32);
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                  const float4 c = __ldg(cs4 + e / 2);  // (cos_e, sin_e, cos_e+1, sin_e+1)
                  float x1 = a[e], x2 = b[e];
                  a[e] = x1 * c.x - x2 * c.y;
                  b[e] = x2 * c.x + x1 * c.y;
                  x1 = a[e + 1];
                  x2 = b[e + 1];
                  a[e + 1] = x1 * c.z - x2 * c.w;
                  b[e + 1] = x2 * c.z + x1 * c.w;
                }
              } else {
#pragma unroll 4
                for (int e = 0; e < 32; ++e) {
                  const float ang = static_cast<float>(pos) * __ldg(p.inv_freq + j * 32 + e);
                  float sn, cs;
                  sincosf(ang, &sn, &cs);
                  const float x1 = a[e], x2 = b[e];
                  a[e] = x1 * cs - x2 * sn;
                  b[e] = x2 * cs + x1 * sn;
                }
              }
            }
            __nv_bfloat16* crow =
                reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(row) * p.ldc;
            store_row32_bf16(crow + col_lo, col_lo, p.N, a);
            store_row32_bf16(crow + col_hi, col_hi, p.N, b);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult qres;
    void* ptr = nullptr;
    cudaError_t err = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                                       cudaEnableDefault, &qres);
    TORCH_CHECK(err == cudaSuccess && qres == cudaDriverEntryPointSuccess && ptr != nullptr,
                "nano_megatron_b200: cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with row pitch `ld`
// elements; box = [box_rows, 64 cols], 128-byte swizzle, zero fill out of bounds.
static CUtensorMap make_tmap_2d(const void* base, int64_t rows, int64_t cols, int64_t ld,
                                int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base),
                               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", static_cast<int>(r),
              ") rows=", rows, " cols=", cols, " ld=", ld);
  return m;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool GATHER = false>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, GemmParams& p,
                   cudaStream_t stream, int max_ctas, const CommMaps* cmp = nullptr) {
  constexpr int smem_bytes = gemm_smem_bytes<BN, EPI>();
  static_assert(smem_bytes <= 227 * 1024, "GEMM shared memory exceeds the per-CTA limit");
  auto kern = gemm_tcgen05_kernel<BN, A_MN, B_MN, EPI, GATHER>;
  static CommMaps empty_maps{};
  const CommMaps& cm = cmp != nullptr ? *cmp : empty_maps;
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes));
    attr_set = true;
  }
  const int tiles = p.num_m_tiles * p.num_n_tiles * p.splits;
  int grid = std::min(tiles, max_ctas > 0 ? max_ctas : num_sms());
  kern<<<grid, gemm_threads<EPI>(), smem_bytes, stream>>>(ta, tb, cm, p); NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static void check_operand(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must have unit inner stride");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0, name, " row pitch must be a multiple of 16 bytes");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name,
              " must be 16-byte aligned");
}

// Dispatch on the run-time layout / epilogue to a compiled instantiation.
template <bool A_MN, bool B_MN, int EPI, bool GATHER = false>
static void dispatch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, GemmParams& p,
                        cudaStream_t s, int max_ctas, const CommMaps* cm = nullptr) {
  if (bn == 256)
    launch<256, A_MN, B_MN, EPI, GATHER>(ta, tb, p, s, max_ctas, cm);
  else
    launch<128, A_MN, B_MN, EPI, GATHER>(ta, tb, p, s, max_ctas, cm);
}

// Split-K factor for an fp32-accumulating GEMM: the smallest split (<= 8, >= 4 K-blocks
// each) that fills the SMs' waves clearly better than no split. Deterministic mode runs
// unsplit: each output tile then has one writer, which adds to C with plain stores.
static int choose_splits(int tiles, int num_kb) {
  if (deterministic_mode()) return 1;
  const int sms = num_sms();
  auto eff = [&](int s) {
    const int work = tiles * s;
    return static_cast<double>(work) / (static_cast<double>((work + sms - 1) / sms) * sms);
  };
  int best = 1;
  double best_eff = eff(1);
  for (int s = 2; s <= 8 && num_kb / s >= 4; ++s) {
    if (eff(s) > best_eff + 0.05) {
      best = s;
      best_eff = eff(s);
    }
  }
  return best;
}

// Pick the N tile. Measured on B200 (bf16 out, M = 4096, N in 1024..8192, K in 1024..2736):
// 128 x 256 tiles beat 128 x 128 tiles at every shape (the MMA issues twice the work per
// instruction for the same A traffic), even when that leaves part of the last wave idle.
// fp32-accumulating weight-gradient GEMMs use 128 x 128 tiles plus split-K instead.
static int choose_bn(int M, int N, int epi) {
  (void)M;
  if (epi == kEpiSwiGLU || epi == kEpiCEStats) return 256;
  if (epi == kEpiF32Acc) return 128;
  return N > 128 ? 256 : 128;
}

}  // namespace nmb

// Python-facing entry points ------------------------------------------------------------

using namespace nmb;

// C = alpha * A.B^T (+R) with layout flags; C dtype bf16 (epi 0/3) or fp32 (epi 1).
// a_mn: `a` holds A as [K, M]; b_mn: `b` holds B as [K, N].
void gemm_tc(at::Tensor a, bool a_mn, at::Tensor b, bool b_mn, at::Tensor c, int64_t epi,
             c10::optional<at::Tensor> residual, c10::optional<at::Tensor> alpha_t, double alpha,
             double beta, c10::optional<at::Tensor> aux, int64_t swiglu_up_row,
             c10::optional<at::Tensor> positions, c10::optional<at::Tensor> inv_freq,
             int64_t head_dim, int64_t rope_cols, int64_t pos_div, at::Tensor status,
             int64_t bn_override, int64_t max_ctas, c10::optional<at::Tensor> rope_cs,
             c10::optional<at::Tensor> ce_part) {
  check_operand(a, "A");
  check_operand(b, "B");
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm_tc: K mismatch ", K, " vs ", Kb);
  TORCH_CHECK(c.dim() == 2 && c.stride(1) == 1 && c.size(0) == M, "gemm_tc: bad C");
  const int64_t N = c.size(1);
  GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.C = c.data_ptr();
  p.ldc = c.stride(0);
  p.alpha = static_cast<float>(alpha);
  p.beta = static_cast<float>(beta);
  p.status = status.data_ptr<int>();
  p.splits = 1;
  if (residual.has_value()) {
    TORCH_CHECK(residual->scalar_type() == at::kBFloat16 && residual->stride(1) == 1);
    p.R = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    p.ldr = residual->stride(0);
  }
  if (alpha_t.has_value()) {
    TORCH_CHECK(alpha_t->scalar_type() == at::kFloat && alpha_t->is_cuda());
    p.alpha_ptr = alpha_t->data_ptr<float>();
  }
  if (epi == kEpiF32Acc) {
    TORCH_CHECK(c.scalar_type() == at::kFloat, "wgrad accumulation output must be fp32");
  } else {
    TORCH_CHECK(c.scalar_type() == at::kBFloat16, "output must be bf16");
  }
  int bn = bn_override > 0 ? static_cast<int>(bn_override) : choose_bn(p.M, p.N, epi);
  if (epi == kEpiSwiGLU) {
    TORCH_CHECK(!a_mn && !b_mn, "SwiGLU epilogue requires K-major operands");
    TORCH_CHECK(aux.has_value(), "SwiGLU epilogue needs the gate|up store");
    p.aux = reinterpret_cast<__nv_bfloat16*>(aux->data_ptr());
    p.ld_aux = aux->stride(0);
    p.swiglu_up_row = static_cast<int>(swiglu_up_row);
    bn = 256;
  }
  if (epi == kEpiCEStats) {
    bn = 256;
    const int64_t parts = ((N + bn - 1) / bn) * kCEPartsPerTile;
    TORCH_CHECK(ce_part.has_value() && ce_part->is_cuda() &&
                    ce_part->scalar_type() == at::kFloat && ce_part->is_contiguous() &&
                    ce_part->numel() >= M * parts * 2,
                "LM-head statistics epilogue needs an fp32 [M, n-tiles x 2, 2] buffer");
    TORCH_CHECK(!a_mn && !b_mn, "LM-head statistics epilogue requires K-major operands");
    p.ce_part = reinterpret_cast<float2*>(ce_part->data_ptr<float>());
  }
  if (epi == kEpiRoPE) {
    TORCH_CHECK(positions.has_value() && inv_freq.has_value(), "RoPE epilogue inputs missing");
    TORCH_CHECK(head_dim == 64 || head_dim == 128, "RoPE epilogue supports head_dim 64/128");
    p.positions = positions->data_ptr<int>();
    p.seq_len = static_cast<int>(positions->numel());
    p.pos_div = static_cast<int>(pos_div > 0 ? pos_div : 1);
    p.inv_freq = inv_freq->data_ptr<float>();
    p.head_dim = static_cast<int>(head_dim);
    p.rope_cols = static_cast<int>(rope_cols);
    TORCH_CHECK(rope_cols % head_dim == 0 && N % head_dim == 0);
    if (rope_cs.has_value()) {
      TORCH_CHECK((rope_cs->scalar_type() == at::kFloat ||
                   rope_cs->scalar_type() == at::kBFloat16) && rope_cs->is_contiguous() &&
                      rope_cs->numel() == positions->numel() * head_dim,
                  "rope table must be fp32 or bf16 [seq_len, head_dim/2, 2]");
      if (rope_cs->scalar_type() == at::kBFloat16)
        p.rope_cs16 = reinterpret_cast<const uint32_t*>(rope_cs->data_ptr());
      else
        p.rope_cs = reinterpret_cast<const float2*>(rope_cs->data_ptr<float>());
    }
  }
  if (epi == kEpiF32Acc && beta == 1.0) {
    bn = bn_override > 0 ? static_cast<int>(bn_override) : 128;
    const int tiles = static_cast<int>(((M + kBM - 1) / kBM) * ((N + bn - 1) / bn));
    p.splits = choose_splits(tiles, static_cast<int>((K + kBK - 1) / kBK));
  }
  const int out_cols_per_tile = epi == kEpiSwiGLU ? bn / 2 : bn;
  p.num_m_tiles = static_cast<int>((M + kBM - 1) / kBM);
  p.num_n_tiles = static_cast<int>((N + out_cols_per_tile - 1) / out_cols_per_tile);
  if (M == 0 || N == 0) return;

  const at::cuda::CUDAGuard guard(a.device());
  ensure_current_context(a.device().index());
  // Tensor maps. A: K-major -> [M, K] with box 128 rows; MN-major -> [K, M] box 64 rows.
  CUtensorMap ta = a_mn ? make_tmap_2d(a.data_ptr(), K, M, a.stride(0), kBK)
                        : make_tmap_2d(a.data_ptr(), M, K, a.stride(0), kBM);
  CUtensorMap tb;
  const int64_t b_rows_total = b_mn ? b.size(1) : b.size(0);
  if (b_mn)
    tb = make_tmap_2d(b.data_ptr(), K, b_rows_total, b.stride(0), kBK);
  else
    tb = make_tmap_2d(b.data_ptr(), b_rows_total, K, b.stride(0),
                      epi == kEpiSwiGLU ? bn / 2 : bn);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int mc = static_cast<int>(max_ctas);
  if (epi == kEpiSwiGLU) {
    launch<256, false, false, kEpiSwiGLU>(ta, tb, p, stream, mc);
  } else if (epi == kEpiRoPE) {
    TORCH_CHECK(!a_mn && !b_mn, "RoPE epilogue requires K-major operands");
    dispatch_bn<false, false, kEpiRoPE>(bn, ta, tb, p, stream, mc);
  } else if (epi == kEpiCEStats) {
    launch<256, false, false, kEpiCEStats>(ta, tb, p, stream, mc);
  } else if (epi == kEpiBF16) {
    if (!a_mn && !b_mn) dispatch_bn<false, false, kEpiBF16>(bn, ta, tb, p, stream, mc);
    else if (!a_mn && b_mn) dispatch_bn<false, true, kEpiBF16>(bn, ta, tb, p, stream, mc);
    else if (a_mn && !b_mn) dispatch_bn<true, false, kEpiBF16>(bn, ta, tb, p, stream, mc);
    else dispatch_bn<true, true, kEpiBF16>(bn, ta, tb, p, stream, mc);
  } else {
    if (!a_mn && !b_mn) dispatch_bn<false, false, kEpiF32Acc>(bn, ta, tb, p, stream, mc);
    else if (!a_mn && b_mn) dispatch_bn<false, true, kEpiF32Acc>(bn, ta, tb, p, stream, mc);
    else if (a_mn && !b_mn) dispatch_bn<true, false, kEpiF32Acc>(bn, ta, tb, p, stream, mc);
    else dispatch_bn<true, true, kEpiF32Acc>(bn, ta, tb, p, stream, mc);
  }
}

// AG -> GEMM: C[M, N] = epilogue(A_gathered . B^T), A_gathered = concat over TP ranks of
// the [R, K] shards at `shard_ptrs[r]` / `shard_ptrs_odd[r]` for an even / odd epoch (row
// pitch `lda`); the epoch is read from `epoch_ptr` (already advanced by this call's
// signal), and rank r's shard is ready once its slot in `flags_ptr` reaches it. With `xfull`, the
// gathered A is also written to that local [M, K] tensor. Epilogues: bf16 (dgrad of a
// row-parallel layer, `b_mn`), RoPE (QKV) or SwiGLU (gate|up).
void gemm_tc_ag(at::Tensor a_local, std::vector<int64_t> shard_ptrs,
                std::vector<int64_t> shard_ptrs_odd, int64_t lda, at::Tensor b, bool b_mn,
                at::Tensor c, int64_t epi, c10::optional<at::Tensor> xfull,
                c10::optional<at::Tensor> aux, int64_t swiglu_up_row,
                c10::optional<at::Tensor> positions, c10::optional<at::Tensor> inv_freq,
                int64_t head_dim, int64_t rope_cols, int64_t pos_div, int64_t rank,
                int64_t flags_ptr, int64_t epoch_ptr, at::Tensor status,
                c10::optional<at::Tensor> rope_cs, c10::optional<at::Tensor> gather_ready,
                c10::optional<at::Tensor> ce_part) {
  check_operand(a_local, "A shard");
  check_operand(b, "B");
  const int tp = static_cast<int>(shard_ptrs.size());
  TORCH_CHECK(tp >= 1 && tp <= kMaxTP, "gemm_tc_ag: 1..8 ranks");
  TORCH_CHECK(rank >= 0 && rank < tp);
  const int64_t R = a_local.size(0), K = a_local.size(1), M = R * tp;
  TORCH_CHECK(R % kBM == 0, "gemm_tc_ag: rows per rank must be a multiple of 128");
  TORCH_CHECK((lda * 2) % 16 == 0 && lda >= K);
  const int64_t Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm_tc_ag: K mismatch");
  TORCH_CHECK(c.dim() == 2 && c.stride(1) == 1 && c.size(0) == M && c.scalar_type() == at::kBFloat16,
              "gemm_tc_ag: bad C");
  TORCH_CHECK(shard_ptrs_odd.size() == shard_ptrs.size());
  for (auto ptr : shard_ptrs) TORCH_CHECK(ptr % 16 == 0, "shard pointers must be 16-byte aligned");
  for (auto ptr : shard_ptrs_odd) TORCH_CHECK(ptr % 16 == 0, "shard pointers must be 16-byte aligned");
  TORCH_CHECK(epoch_ptr % 4 == 0 && epoch_ptr != 0);
  const int64_t N = c.size(1);
  GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.C = c.data_ptr();
  p.ldc = c.stride(0);
  p.alpha = 1.0f;
  p.status = status.data_ptr<int>();
  p.comm_rows = static_cast<int>(R);
  p.comm_rank = static_cast<int>(rank);
  p.comm_size = tp;
  p.flags = reinterpret_cast<const uint32_t*>(flags_ptr);
  p.epoch_ptr = reinterpret_cast<const uint32_t*>(epoch_ptr);
  p.m_rotate = static_cast<int>(rank * (R / kBM));
  p.splits = 1;
  int bn = choose_bn(p.M, p.N, epi);
  if (epi == kEpiSwiGLU) {
    TORCH_CHECK(!b_mn && aux.has_value());
    p.aux = reinterpret_cast<__nv_bfloat16*>(aux->data_ptr());
    p.ld_aux = aux->stride(0);
    p.swiglu_up_row = static_cast<int>(swiglu_up_row);
    bn = 256;
  } else if (epi == kEpiRoPE) {
    TORCH_CHECK(!b_mn && positions.has_value() && inv_freq.has_value());
    TORCH_CHECK(head_dim == 64 || head_dim == 128);
    p.positions = positions->data_ptr<int>();
    p.seq_len = static_cast<int>(positions->numel());
    p.pos_div = static_cast<int>(pos_div > 0 ? pos_div : 1);
    p.inv_freq = inv_freq->data_ptr<float>();
    p.head_dim = static_cast<int>(head_dim);
    p.rope_cols = static_cast<int>(rope_cols);
    if (rope_cs.has_value()) {
      TORCH_CHECK((rope_cs->scalar_type() == at::kFloat ||
                   rope_cs->scalar_type() == at::kBFloat16) && rope_cs->is_contiguous() &&
                  rope_cs->numel() == positions->numel() * head_dim);
      if (rope_cs->scalar_type() == at::kBFloat16)
        p.rope_cs16 = reinterpret_cast<const uint32_t*>(rope_cs->data_ptr());
      else
        p.rope_cs = reinterpret_cast<const float2*>(rope_cs->data_ptr<float>());
    }
  } else if (epi == kEpiCEStats) {
    bn = 256;
    const int64_t parts = ((N + bn - 1) / bn) * kCEPartsPerTile;
    TORCH_CHECK(!b_mn && ce_part.has_value() && ce_part->is_cuda() &&
                    ce_part->scalar_type() == at::kFloat && ce_part->is_contiguous() &&
                    ce_part->numel() >= M * parts * 2,
                "gemm_tc_ag: LM-head statistics need an fp32 [M, n-tiles x 2, 2] buffer");
    p.ce_part = reinterpret_cast<float2*>(ce_part->data_ptr<float>());
  } else {
    TORCH_CHECK(epi == kEpiBF16, "gemm_tc_ag: epilogue must be bf16, RoPE or SwiGLU");
  }
  const int out_cols = epi == kEpiSwiGLU ? bn / 2 : bn;
  p.num_m_tiles = static_cast<int>(M / kBM);
  p.num_n_tiles = static_cast<int>((N + out_cols - 1) / out_cols);
  if (M == 0 || N == 0) return;
  const at::cuda::CUDAGuard guard(a_local.device());
  ensure_current_context(a_local.device().index());
  CommMaps cm{};
  for (int r = 0; r < tp; ++r) {
    cm.a[0][r] = make_tmap_2d(reinterpret_cast<const void*>(shard_ptrs[r]), R, K, lda, kBM);
    cm.a[1][r] = make_tmap_2d(reinterpret_cast<const void*>(shard_ptrs_odd[r]), R, K, lda, kBM);
  }
  if (xfull.has_value()) {
    check_operand(*xfull, "xfull");
    TORCH_CHECK(xfull->size(0) == M && xfull->size(1) == K);
    cm.xfull = make_tmap_2d(xfull->data_ptr(), M, K, xfull->stride(0), kBM);
    p.store_gathered = 1;
    if (gather_ready.has_value()) {
      TORCH_CHECK(gather_ready->is_cuda() && gather_ready->scalar_type() == at::kInt &&
                      gather_ready->is_contiguous() && gather_ready->numel() >= M / kBM,
                  "gemm_tc_ag: gather_ready must hold one int32 per 128-row tile");
      p.gather_ready = reinterpret_cast<uint32_t*>(gather_ready->data_ptr<int>());
    }
  }
  const int64_t b_rows = b_mn ? b.size(1) : b.size(0);
  CUtensorMap tb = b_mn ? make_tmap_2d(b.data_ptr(), K, b_rows, b.stride(0), kBK)
                        : make_tmap_2d(b.data_ptr(), b_rows, K, b.stride(0),
                                       epi == kEpiSwiGLU ? bn / 2 : bn);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const CUtensorMap& ta = cm.a[0][rank];
  if (epi == kEpiSwiGLU)
    launch<256, false, false, kEpiSwiGLU, true>(ta, tb, p, stream, 0, &cm);
  else if (epi == kEpiRoPE)
    dispatch_bn<false, false, kEpiRoPE, true>(bn, ta, tb, p, stream, 0, &cm);
  else if (epi == kEpiCEStats)
    launch<256, false, false, kEpiCEStats, true>(ta, tb, p, stream, 0, &cm);
  else if (b_mn)
    dispatch_bn<false, true, kEpiBF16, true>(bn, ta, tb, p, stream, 0, &cm);
  else
    dispatch_bn<false, false, kEpiBF16, true>(bn, ta, tb, p, stream, 0, &cm);
}

// GEMM -> RS: partial C = A . B^T for all M rows; row r's bf16 partial goes to rank
// (r / rows_per_rank)'s staging buffer (`staging_ptrs` / `staging_ptrs_odd` by the parity
// of the upcoming epoch, *epoch_ptr + 1), laid out [tp][rows][N] with this rank's slot
// `rank`. The owner reduces the slots with rs_reduce after the signal.
void gemm_tc_rs(at::Tensor a, bool a_mn, at::Tensor b, bool b_mn,
                std::vector<int64_t> staging_ptrs, std::vector<int64_t> staging_ptrs_odd,
                int64_t rows_per_rank, int64_t n_out, int64_t rank, int64_t epoch_ptr,
                at::Tensor status, c10::optional<at::Tensor> alpha_t,
                c10::optional<at::Tensor> out, c10::optional<at::Tensor> residual,
                std::vector<int64_t> tile_flag_ptrs) {
  check_operand(a, "A");
  check_operand(b, "B");
  const int tp = static_cast<int>(staging_ptrs.size());
  TORCH_CHECK(tp >= 1 && tp <= kMaxTP && rank >= 0 && rank < tp);
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  TORCH_CHECK(K == (b_mn ? b.size(0) : b.size(1)), "gemm_tc_rs: K mismatch");
  TORCH_CHECK(M == rows_per_rank * tp, "gemm_tc_rs: M must equal tp * rows_per_rank");
  TORCH_CHECK(rows_per_rank % kBM == 0, "gemm_tc_rs: rows per rank must be a multiple of 128");
  TORCH_CHECK((n_out * 2) % 16 == 0, "gemm_tc_rs: N must be a multiple of 8");
  TORCH_CHECK(staging_ptrs_odd.size() == staging_ptrs.size());
  for (auto ptr : staging_ptrs) TORCH_CHECK(ptr % 16 == 0, "staging must be 16-byte aligned");
  for (auto ptr : staging_ptrs_odd) TORCH_CHECK(ptr % 16 == 0, "staging must be 16-byte aligned");
  TORCH_CHECK(epoch_ptr % 4 == 0 && epoch_ptr != 0);
  GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(n_out);
  p.K = static_cast<int>(K);
  p.ldc = n_out;
  p.alpha = 1.0f;
  p.status = status.data_ptr<int>();
  p.comm_rows = static_cast<int>(rows_per_rank);
  p.comm_rank = static_cast<int>(rank);
  p.comm_size = tp;
  p.splits = 1;
  p.epoch_ptr = reinterpret_cast<const uint32_t*>(epoch_ptr);
  if (alpha_t.has_value()) {
    TORCH_CHECK(alpha_t->is_cuda() && alpha_t->scalar_type() == at::kFloat,
                "gemm_tc_rs: alpha must be an fp32 device scalar");
    p.alpha_ptr = alpha_t->data_ptr<float>();
  }
  for (int r = 0; r < tp; ++r) {
    p.peer_out[0][r] = reinterpret_cast<__nv_bfloat16*>(staging_ptrs[r]);
    p.peer_out[1][r] = reinterpret_cast<__nv_bfloat16*>(staging_ptrs_odd[r]);
  }
  const int bn = choose_bn(p.M, p.N, kEpiPeer);
  p.num_m_tiles = static_cast<int>((M + kBM - 1) / kBM);
  p.num_n_tiles = static_cast<int>((n_out + bn - 1) / bn);
  if (out.has_value()) {
    // reduction in the epilogue: this rank's rows land in `out` (+ residual)
    TORCH_CHECK(static_cast<int>(tile_flag_ptrs.size()) == tp,
                "gemm_tc_rs: one tile-flag array per rank");
    TORCH_CHECK(out->is_cuda() && out->scalar_type() == at::kBFloat16 && out->dim() == 2 &&
                    out->size(0) == rows_per_rank && out->size(1) == n_out &&
                    out->stride(1) == 1 && out->stride(0) % 8 == 0 &&
                    reinterpret_cast<uintptr_t>(out->data_ptr()) % 16 == 0,
                "gemm_tc_rs: out must be a [rows_per_rank, N] bf16 matrix, 16-byte rows");
    TORCH_CHECK((rows_per_rank / kBM) * p.num_n_tiles <= kRsTileFlags,
                "gemm_tc_rs: more tiles than the flag array holds");
    p.rs_inplace = 1;
    p.own_out = reinterpret_cast<__nv_bfloat16*>(out->data_ptr());
    p.ld_own = out->stride(0);
    for (int r = 0; r < tp; ++r) {
      TORCH_CHECK(tile_flag_ptrs[r] % 16 == 0 && tile_flag_ptrs[r] != 0);
      p.tile_flags[r] = reinterpret_cast<uint32_t*>(tile_flag_ptrs[r]);
    }
    if (residual.has_value()) {
      TORCH_CHECK(residual->scalar_type() == at::kBFloat16 && residual->dim() == 2 &&
                      residual->size(0) == rows_per_rank && residual->size(1) == n_out &&
                      residual->stride(1) == 1 && residual->stride(0) % 8 == 0 &&
                      reinterpret_cast<uintptr_t>(residual->data_ptr()) % 16 == 0,
                  "gemm_tc_rs: residual must match out");
      p.R = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
      p.ldr = residual->stride(0);
    }
  }
  if (M == 0 || n_out == 0) return;
  const at::cuda::CUDAGuard guard(a.device());
  ensure_current_context(a.device().index());
  CUtensorMap ta = a_mn ? make_tmap_2d(a.data_ptr(), K, M, a.stride(0), kBK)
                        : make_tmap_2d(a.data_ptr(), M, K, a.stride(0), kBM);
  const int64_t b_rows = b_mn ? b.size(1) : b.size(0);
  CUtensorMap tb = b_mn ? make_tmap_2d(b.data_ptr(), K, b_rows, b.stride(0), kBK)
                        : make_tmap_2d(b.data_ptr(), b_rows, K, b.stride(0), bn);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(!a_mn, "gemm_tc_rs: A must be K-major");
  if (b_mn)
    dispatch_bn<false, true, kEpiPeer>(bn, ta, tb, p, stream, 0);
  else
    dispatch_bn<false, false, kEpiPeer>(bn, ta, tb, p, stream, 0);
}

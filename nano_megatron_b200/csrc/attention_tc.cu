// Causal flash-attention forward on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// One CTA per (128-query block, head, batch); 192 threads:
//   warp 0    : TMA producer — Q once, then K_j / V_j tiles of 128 keys into a
//               2-stage ring (separate K and V barriers so S = Q K^T can start
//               before V lands);
//   warp 1    : TMEM allocator + MMA issuer — S_j = Q K_j^T into TMEM columns
//               [0,128), then O += P_{j-1} V_{j-1} into columns [128, 128+D);
//   warps 2-5 : softmax — each thread owns one query row (one TMEM lane): it
//               loads its S row with tcgen05.ld, releases S at once (so the
//               next QK^T overlaps the exponentials), computes the online
//               softmax in base 2, rescales its O row in TMEM when the running
//               max grows, writes P (bf16) to shared memory in the UMMA
//               K-major 128-byte-swizzled layout and signals the MMA warp;
//               at the end it normalises O and stores O and the base-2 LSE;
//   warp 6    : ring pull (context parallelism) — copies this CTA's slice of the
//               next ring step's K/V block from the owner GPU's memory into a local
//               buffer while the other warps compute (idle otherwise).
// Q/K/V are read through 4-D TMA maps (d, head, seq, batch) over the strided
// views of the fused QKV buffer; P is the A operand (K-major) and V the B
// operand (MN-major) of the second product. Causal key blocks above the
// diagonal are skipped; rows of the diagonal / tail block are masked.
//
// Same contract and numerics as flash_attn_fwd (attention.cu): base-2 LSE.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace nmb {
namespace fatc {

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kThreads = 224;      // 6 compute warps + 1 pull warp
constexpr int kPullWarp = 6;
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct Cfg {
  static constexpr int kQBytes = kBM * D * 2;
  static constexpr int kKBytes = kBN * D * 2;
  static constexpr int kVBytes = kBN * D * 2;
  static constexpr int kPBytes = kBM * kBN * 2;
  static constexpr int kStages = 2;
  static constexpr int kSmem = kQBytes + kStages * (kKBytes + kVBytes) + kPBytes + 1024 + 256;
  static constexpr int kTmemCols = 256;  // S: [0,128), O: [128, 128+D)
};

struct Params {
  __nv_bfloat16* o;
  int64_t o_row, o_batch;
  float* lse;
  int B, Hq, Hkv, Sq, Sk;
  int q_offset, k_offset;
  int causal;
  float scale_log2;
  int* status;
  PullDesc pull;
};

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

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const Params p) {
  using C = Cfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::kQBytes;
  uint8_t* sV = sK + C::kStages * C::kKBytes;
  uint8_t* sP = sV + C::kStages * C::kVBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + C::kPBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;
  uint64_t* s_free = bars + 10;
  uint64_t* p_full = bars + 11;
  uint64_t* o_done = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int mblk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.Hq / p.Hkv);
  const int m0 = mblk * kBM;
  const int warp = threadIdx.x / 32;
  int n_end = p.Sk;
  if (p.causal) {
    const int last_q = p.q_offset + min(m0 + kBM, p.Sq) - 1;
    n_end = min(p.Sk, last_q - p.k_offset + 1);
  }
  const int nblk = n_end > 0 ? (n_end + kBN - 1) / kBN : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem;
  const uint32_t tO = tmem + 128;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (elect_one() && nblk > 0) {
      mbar_arrive_expect_tx(q_full, C::kQBytes);
#pragma unroll
      for (int c = 0; c < D / 64; ++c)
        tma_load_4d(sQ + c * kBM * 128, &tmQ, q_full, c * 64, h, m0, b);
      for (int j = 0; j < nblk; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_empty[st], ph ^ 1u, p.status, kStatusAttnTimeout, abort_flag)) break;
        mbar_arrive_expect_tx(&k_full[st], C::kKBytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sK + st * C::kKBytes + c * kBN * 128, &tmK, &k_full[st], c * 64, kvh,
                      j * kBN, b);
        if (!mbar_wait(&v_empty[st], ph ^ 1u, p.status, kStatusAttnTimeout, abort_flag)) break;
        mbar_arrive_expect_tx(&v_full[st], C::kVBytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sV + st * C::kVBytes + c * kBN * 128, &tmV, &v_full[st], c * 64, kvh,
                      j * kBN, b);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (elect_one() && nblk > 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kBM, kBN, false, false);
      constexpr uint32_t idesc_o = umma_idesc_bf16(kBM, D, false, true);
      bool ok = mbar_wait(q_full, 0, p.status, kStatusAttnTimeout, abort_flag);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t p_addr = smem_u32(sP);
      auto do_pv = [&](int i) -> bool {
        const int st = i & 1;
        if (!mbar_wait(p_full, i & 1, p.status, kStatusAttnTimeout, abort_flag)) return false;
        if (!mbar_wait(&v_full[st], (i >> 1) & 1, p.status, kStatusAttnTimeout, abort_flag))
          return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + st * C::kVBytes);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t ad = umma_desc_sw128(p_addr + (kk >> 2) * (kBM * 128) + (kk & 3) * 32,
                                              16, 1024);
          const uint64_t bd = umma_desc_sw128(v_addr + kk * 2048, kBN * 128, 1024);
          umma_f16_ss(tO, ad, bd, idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(o_done);
        umma_commit(&v_empty[st]);
        return true;
      };
      for (int j = 0; j < nblk && ok; ++j) {
        const int st = j & 1;
        ok = mbar_wait(&k_full[st], (j >> 1) & 1, p.status, kStatusAttnTimeout, abort_flag);
        if (ok && j > 0) ok = mbar_wait(s_free, (j - 1) & 1, p.status, kStatusAttnTimeout,
                                        abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * C::kKBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (kBM * 128) + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * (kBN * 128) + (kk & 3) * 32;
          umma_f16_ss(tS, umma_desc_sw128(q_addr + off, 16, 1024),
                      umma_desc_sw128(k_addr + koff, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        umma_commit(&k_empty[st]);
        if (j > 0) ok = do_pv(j - 1);
      }
      if (ok) do_pv(nblk - 1);
    }
  } else if (warp == kPullWarp) {
    pull_slice(p.pull, threadIdx.x & 31, 32);
  } else {
    // ---------------------------------------------------------------- softmax
    const int quarter = warp & 3;
    const int lane = threadIdx.x & 31;
    const int row = quarter * 32 + lane;  // row inside the block == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int qpos = p.q_offset + m0 + row;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk && ok; ++j) {
      ok = mbar_wait(s_full, j & 1, p.status, kStatusAttnTimeout, abort_flag);
      if (!ok) break;
      tc_fence_after();
      // all four 32-column loads in flight together, one wait
      uint32_t r[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c)
        tmem_ld_32x32b_x32(tS + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(r + c * 32));
      tmem_wait_ld();
      float s[kBN];
#pragma unroll
      for (int e = 0; e < kBN; ++e) s[e] = __uint_as_float(r[e]) * p.scale_log2;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      const int n0 = j * kBN;
      const bool need_mask = (n0 + kBN > p.Sk) ||
                             (p.causal && p.k_offset + n0 + kBN - 1 > p.q_offset + m0);
      if (need_mask) {
        // visible keys of this query row in the block: columns [0, vis), applied with a
        // select per element (per-element compare-and-branch stalled the phase)
        int vis = min(kBN, p.Sk - n0);
        if (p.causal) vis = min(vis, qpos - p.k_offset - n0 + 1);
#pragma unroll
        for (int e = 0; e < kBN; ++e) s[e] = e < vis ? s[e] : -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < kBN; ++e) mx = fmaxf(mx, s[e]);
      const float m_new = fmaxf(m_run, mx);
      const float corr = (m_run == -INFINITY) ? 0.f : ex2(m_run - m_new);
      float rs = 0.f;
      uint32_t pk[kBN / 2];
      // a row with no visible key yet (m_new = -inf) has s = -inf everywhere: exponent
      // reference 0 gives P = 0 without a per-element test
      const float mref = m_new == -INFINITY ? 0.f : m_new;
#pragma unroll
      for (int e = 0; e < kBN; ++e) s[e] = ex2(s[e] - mref);
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};   // four partial sums: short dependency chains
#pragma unroll
      for (int e = 0; e < kBN; e += 2) {
        rs4[(e / 2) & 3] += s[e] + s[e + 1];
        pk[e / 2] = pack_bf16x2(s[e], s[e + 1]);
      }
      rs = (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      l_run = l_run * corr + rs;
      // PV_{j-1} must be complete before P is overwritten or O is rescaled.
      if (j > 0) {
        ok = mbar_wait(o_done, (j - 1) & 1, p.status, kStatusAttnTimeout, abort_flag);
        if (!ok) break;
        tc_fence_after();
        // tcgen05.ld/st are warp-collective: decide the rescale per warp (rows
        // whose max did not grow get corr == 1; rows with no mass yet have O == 0).
        const bool grow = m_new > m_run && m_run != -INFINITY;
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tO + lane_off + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * corr);
            tmem_st_32x32b_x32(tO + lane_off + c * 32, r);
          }
          tmem_wait_st();
        }
      }
      m_run = m_new;
      // P row -> shared memory, UMMA K-major SW128 layout (two 64-column atoms).
#pragma unroll
      for (int ch = 0; ch < kBN / 8; ++ch) {
        const int atom = ch >> 3, c8 = ch & 7;
        uint8_t* dst = sP + atom * (kBM * 128) + row * 128 + ((c8 ^ (row & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) =
            make_uint4(pk[ch * 4 + 0], pk[ch * 4 + 1], pk[ch * 4 + 2], pk[ch * 4 + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // epilogue
    if (ok && nblk > 0 &&
        mbar_wait(o_done, (nblk - 1) & 1, p.status, kStatusAttnTimeout, abort_flag)) {
      tc_fence_after();
      const int grow = m0 + row;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* orow = p.o + b * p.o_batch + static_cast<int64_t>(grow) * p.o_row +
                            static_cast<int64_t>(h) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tO + lane_off + c * 32, r);
        tmem_wait_ld();
        if (grow < p.Sq) {
          uint4* d4 = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            d4[q] = make_uint4(pack_bf16x2(__uint_as_float(r[q * 8 + 0]) * inv,
                                           __uint_as_float(r[q * 8 + 1]) * inv),
                               pack_bf16x2(__uint_as_float(r[q * 8 + 2]) * inv,
                                           __uint_as_float(r[q * 8 + 3]) * inv),
                               pack_bf16x2(__uint_as_float(r[q * 8 + 4]) * inv,
                                           __uint_as_float(r[q * 8 + 5]) * inv),
                               pack_bf16x2(__uint_as_float(r[q * 8 + 6]) * inv,
                                           __uint_as_float(r[q * 8 + 7]) * inv));
        }
      }
      if (grow < p.Sq)
        p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.Sq + grow] =
            l_run > 0.f ? m_run + __log2f(l_run) : -INFINITY;
    } else if (nblk == 0) {
      // no visible key: output zeros, LSE -inf
      const int grow = m0 + row;
      if (grow < p.Sq) {
        __nv_bfloat16* orow = p.o + b * p.o_batch + static_cast<int64_t>(grow) * p.o_row +
                              static_cast<int64_t>(h) * D;
        for (int d = 0; d < D; ++d) orow[d] = __float2bfloat16_rn(0.f);
        p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.Sq + grow] = -INFINITY;
      }
    }
  }
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

// 4-D map over a [B, S, H, D] strided bf16 view: dims (d, h, s, b), box (64, 1, rows, 1).
static CUtensorMap make_map(const at::Tensor& t, int rows) {
  CUtensorMap m;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(t.size(3)), static_cast<cuuint64_t>(t.size(2)),
                        static_cast<cuuint64_t>(t.size(1)), static_cast<cuuint64_t>(t.size(0))};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(t.stride(2) * 2),
                           static_cast<cuuint64_t>(t.stride(1) * 2),
                           static_cast<cuuint64_t>(t.stride(0) * 2)};
  cuuint32_t box[4] = {64u, 1u, static_cast<cuuint32_t>(rows), 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, t.data_ptr(), dims, strides,
                           box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "flash_attn_fwd_tc: tensor map encode failed (", (int)r, ")");
  return m;
}

}  // namespace fatc
}  // namespace nmb

using namespace nmb;
using namespace nmb::fatc;

// Ring-pull descriptor from host arguments (pull_src == 0: no pull).
PullDesc make_pull(int64_t src, const c10::optional<at::Tensor>& dst, int64_t flag, int64_t epoch,
                   int* status) {
  PullDesc d{};
  if (src == 0) return d;
  TORCH_CHECK(dst.has_value() && dst->is_cuda() && dst->is_contiguous() &&
                  dst->nbytes() % 16 == 0 && reinterpret_cast<uintptr_t>(dst->data_ptr()) % 16 == 0,
              "ring pull: destination must be a contiguous, 16-byte multiple CUDA buffer");
  TORCH_CHECK(src % 16 == 0 && flag % 4 == 0 && flag != 0 && epoch % 4 == 0 && epoch != 0,
              "ring pull: bad source / flag / epoch address");
  d.src = reinterpret_cast<const uint4*>(src);
  d.dst = reinterpret_cast<uint4*>(dst->data_ptr());
  d.vec16 = static_cast<long long>(dst->nbytes() / 16);
  d.flag = reinterpret_cast<const uint32_t*>(flag);
  d.epoch_ptr = reinterpret_cast<const uint32_t*>(epoch);
  d.status = status;
  return d;
}

// Same contract as flash_attn_fwd; runs the tcgen05 kernel.
void flash_attn_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse,
                       double softmax_scale, bool causal, int64_t q_offset, int64_t k_offset,
                       at::Tensor status, int64_t pull_src, c10::optional<at::Tensor> pull_dst,
                       int64_t pull_flag, int64_t pull_epoch) {
  const int64_t D = q.size(3);
  TORCH_CHECK(D == 64 || D == 128, "flash_attn_fwd_tc: head_dim must be 64 or 128");
  for (const at::Tensor* t : {&q, &k, &v, &o}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 4);
    TORCH_CHECK(t->stride(3) == 1 && t->stride(2) == D, "heads must be contiguous [.., H, D]");
    TORCH_CHECK(t->stride(1) % 8 == 0 && t->stride(0) % 8 == 0, "strides must be 16-byte");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0, "16-byte alignment");
  }
  Params p{};
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.o_row = o.stride(1);
  p.o_batch = o.stride(0);
  p.lse = lse.data_ptr<float>();
  p.B = q.size(0);
  p.Sq = q.size(1);
  p.Hq = q.size(2);
  p.Sk = k.size(1);
  p.Hkv = k.size(2);
  TORCH_CHECK(p.Hq % p.Hkv == 0);
  p.q_offset = q_offset;
  p.k_offset = k_offset;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = static_cast<float>(softmax_scale) * kLog2e;
  p.status = status.data_ptr<int>();
  p.pull = make_pull(pull_src, pull_dst, pull_flag, pull_epoch, p.status);
  if (p.B == 0 || p.Sq == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  ensure_current_context(q.device().index());
  CUtensorMap mq = make_map(q, kBM), mk = make_map(k, kBN), mv = make_map(v, kBN);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  dim3 grid((p.Sq + kBM - 1) / kBM, p.Hq, p.B);
  if (D == 64) {
    static bool set = false;
    if (!set) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(flash_fwd_tc_kernel<64>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          Cfg<64>::kSmem));
      set = true;
    }
    flash_fwd_tc_kernel<64><<<grid, kThreads, Cfg<64>::kSmem, stream>>>(mq, mk, mv, p);
  } else {
    static bool set = false;
    if (!set) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(flash_fwd_tc_kernel<128>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          Cfg<128>::kSmem));
      set = true;
    }
    flash_fwd_tc_kernel<128><<<grid, kThreads, Cfg<128>::kSmem, stream>>>(mq, mk, mv, p);
  }
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Tensor-parallel embedding and cross-entropy collectives over NVLink peer memory.
//
// Embedding forward (lookup fused with the sequence-parallel reduce-scatter). The
// vocabulary is split over the TP ranks and every token id belongs to exactly one of
// them, so the "sum over ranks" of the partial lookups is a selection: each rank looks
// up only the tokens whose id falls in its shard and stores each such row straight into
// the symmetric slot of the rank that owns the token's sequence position (local store
// or peer store). Every output row is written exactly once; the owner waits (bounded)
// for every rank's flag and copies its slot out. No partial [T, H] tensor, no reduction.
//
// Embedding backward (all-gather fused with the scatter-add): every rank publishes its
// dY shard (the existing AG slot); each rank then walks all tokens, and for those whose
// id lies in its vocabulary shard reads the dY row from the owner's slot (peer load)
// and adds it into its fp32 gradient rows. Only 1/TP of the rows cross NVLink per rank.
//
// Cross-entropy statistics (C6): each rank's per-row (max, sum-exp, target logit) of its
// vocabulary shard is stored into slot [this rank] of every TP rank's statistics buffer
// (peer stores); after a signal, the finish kernel waits for every rank's flag and merges
// the TP slots in-kernel into the loss and the in-place softmax - onehot gradient.
//
// Slots alternate by the parity of the channel's device epoch (advanced by the signal
// kernel), so consecutive calls never overwrite data a peer may still read; every wait
// is bounded and records 0x301 in the status word on expiry.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace nmb {

constexpr int kAuxMaxTP = 8;
constexpr float kLog2eAux = 1.4426950408889634f;
constexpr float kLn2Aux = 0.6931471805599453f;

struct AuxPtrs {
  void* even[kAuxMaxTP];   // per rank, slot of an even epoch
  void* odd[kAuxMaxTP];    // per rank, slot of an odd epoch
};

__device__ __forceinline__ uint32_t read_epoch(const uint32_t* epoch_ptr) {
  return *reinterpret_cast<const volatile uint32_t*>(epoch_ptr);
}

// Thread 0 of each block waits until every rank's flag reached the current epoch; the
// block's answer lands in *ok (shared).
__device__ __forceinline__ void block_wait_flags(const uint32_t* flags, int n,
                                                 const uint32_t* epoch_ptr, int* status,
                                                 int* ok) {
  if (threadIdx.x == 0) {
    const uint32_t e = read_epoch(epoch_ptr);
    int good = 1;
    for (int r = 0; r < n && good; ++r)
      good = wait_flag(flags + r, e, status, kStatusPeerFlagTimeout, nullptr) ? 1 : 0;
    *ok = good;
  }
  __syncthreads();
}

// ------------------------------------------------------------------ embedding forward
// ids: [T] (every token of the TP group's sequence block, sequence-major); w: this rank's
// [V, H] shard starting at vocabulary row vstart. Token t belongs to rank t / R.
__global__ void embedding_scatter_kernel(const int64_t* __restrict__ ids,
                                         const __nv_bfloat16* __restrict__ w, int64_t V,
                                         int64_t vstart, int T, int H, int R, AuxPtrs dst,
                                         const uint32_t* epoch_ptr) {
  const uint32_t e = read_epoch(epoch_ptr) + 1u;   // the signal that follows advances it
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x / 32;
  const int nvec = H / 8;
  for (int t = blockIdx.x * warps + threadIdx.x / 32; t < T; t += gridDim.x * warps) {
    const int64_t id = ids[t] - vstart;
    if (id < 0 || id >= V) continue;
    const int owner = t / R;
    __nv_bfloat16* slot = static_cast<__nv_bfloat16*>((e & 1u) ? dst.odd[owner]
                                                                : dst.even[owner]);
    uint4* o = reinterpret_cast<uint4*>(slot + static_cast<int64_t>(t - owner * R) * H);
    const uint4* src = reinterpret_cast<const uint4*>(w + id * H);
    for (int c = lane; c < nvec; c += 32) o[c] = src[c];
  }
}

// out[R, H] = this rank's slot of the current epoch, once every rank has signalled.
__global__ void embedding_collect_kernel(const __nv_bfloat16* even, const __nv_bfloat16* odd,
                                         __nv_bfloat16* __restrict__ out, int64_t ldo, int R,
                                         int H, const uint32_t* flags, int tp,
                                         const uint32_t* epoch_ptr, int* status) {
  __shared__ int ok;
  block_wait_flags(flags, tp, epoch_ptr, status, &ok);
  if (!ok) return;
  const __nv_bfloat16* src = (read_epoch(epoch_ptr) & 1u) ? odd : even;
  const int nvec = H / 8;
  const int64_t total = static_cast<int64_t>(R) * nvec;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nvec, c = i - r * nvec;
    reinterpret_cast<uint4*>(out + r * ldo)[c] =
        __ldcg(reinterpret_cast<const uint4*>(src + r * H) + c);
  }
}

// ------------------------------------------------------------------ embedding backward
// dY of token t lives in rank (t / R)'s AG slot (current epoch), row t % R, pitch H.
__global__ void embedding_bwd_gather_kernel(const int64_t* __restrict__ ids, AuxPtrs src,
                                            float* __restrict__ grad, int64_t V,
                                            int64_t vstart, int T, int H, int R,
                                            const uint32_t* flags, int tp,
                                            const uint32_t* epoch_ptr, int* status) {
  __shared__ int ok;
  block_wait_flags(flags, tp, epoch_ptr, status, &ok);
  if (!ok) return;
  const bool odd = read_epoch(epoch_ptr) & 1u;
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x / 32;
  const int nvec = H / 8;
  for (int t = blockIdx.x * warps + threadIdx.x / 32; t < T; t += gridDim.x * warps) {
    const int64_t id = ids[t] - vstart;
    if (id < 0 || id >= V) continue;
    const int owner = t / R;
    const __nv_bfloat16* row =
        static_cast<const __nv_bfloat16*>(odd ? src.odd[owner] : src.even[owner]) +
        static_cast<int64_t>(t - owner * R) * H;
    float* dst = grad + id * H;
    for (int c = lane; c < nvec; c += 32) {
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(row) + c);
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
      float f[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        f[2 * j] = bf16_lo(wv[j]);
        f[2 * j + 1] = bf16_hi(wv[j]);
      }
      asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + c * 8),
                   "f"(f[0]), "f"(f[1]), "f"(f[2]), "f"(f[3])
                   : "memory");
      asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + c * 8 + 4),
                   "f"(f[4]), "f"(f[5]), "f"(f[6]), "f"(f[7])
                   : "memory");
    }
  }
}

// Deterministic variant (deterministic_mode()): tokens stably sorted by id, each run of
// equal ids added in token order by one warp (add_sorted_runs), after the same flag wait.
struct GatheredRows {
  AuxPtrs src;
  bool odd;
  int R, H;
  __device__ __forceinline__ uint4 operator()(int64_t t, int c) const {
    const int owner = static_cast<int>(t / R);
    const __nv_bfloat16* row =
        static_cast<const __nv_bfloat16*>(odd ? src.odd[owner] : src.even[owner]) +
        (t - static_cast<int64_t>(owner) * R) * H;
    return __ldcg(reinterpret_cast<const uint4*>(row) + c);
  }
};

__global__ void embedding_bwd_gather_sorted_kernel(const int64_t* __restrict__ sorted_ids,
                                                   const int64_t* __restrict__ order,
                                                   AuxPtrs src, float* __restrict__ grad,
                                                   int64_t V, int64_t vstart, int T, int H,
                                                   int R, const uint32_t* flags, int tp,
                                                   const uint32_t* epoch_ptr, int* status) {
  __shared__ int ok;
  block_wait_flags(flags, tp, epoch_ptr, status, &ok);
  if (!ok) return;
  const bool odd = read_epoch(epoch_ptr) & 1u;
  add_sorted_runs(sorted_ids, order, T, vstart, V, H, grad, GatheredRows{src, odd, R, H});
}

// ------------------------------------------------------------------ cross-entropy
__device__ __forceinline__ float ex2_aux(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Online (max, sum of exp) of one bf16 row, reduced over the block.
template <int NT>
__device__ void row_stats(const __nv_bfloat16* row, int V, float& m_out, float& s_out) {
  float m = -INFINITY, s = 0.f;
  const int nvec = V / 8;
  for (int c = threadIdx.x; c < nvec; c += NT) {
    const uint4 v = reinterpret_cast<const uint4*>(row)[c];
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float x = h ? bf16_hi(wv[j]) : bf16_lo(wv[j]);
        if (x > m) {
          s = (m == -INFINITY ? 0.f : s * ex2_aux((m - x) * kLog2eAux)) + 1.f;
          m = x;
        } else {
          s += ex2_aux((x - m) * kLog2eAux);
        }
      }
    }
  }
  __shared__ float red_m[NT / 32], red_s[NT / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * ex2_aux((m - nm) * kLog2eAux)) +
        (om == -INFINITY ? 0.f : os * ex2_aux((om - nm) * kLog2eAux));
    m = nm;
  }
  if ((threadIdx.x & 31) == 0) {
    red_m[threadIdx.x / 32] = m;
    red_s[threadIdx.x / 32] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = red_m[0], S = red_s[0];
    for (int i = 1; i < NT / 32; ++i) {
      const float nm = fmaxf(M, red_m[i]);
      S = (M == -INFINITY ? 0.f : S * ex2_aux((M - nm) * kLog2eAux)) +
          (red_m[i] == -INFINITY ? 0.f : red_s[i] * ex2_aux((red_m[i] - nm) * kLog2eAux));
      M = nm;
    }
    red_m[0] = M;
    red_s[0] = S;
  }
  __syncthreads();
  m_out = red_m[0];
  s_out = red_s[0];
}

// One block per row: (max, sum-exp, target logit) of this rank's vocabulary shard, stored
// into slot [rank] of every TP rank's statistics buffer ([tp][T][3] fp32 per parity).
template <int NT>
__global__ void __launch_bounds__(NT) ce_stats_scatter_kernel(
    const __nv_bfloat16* __restrict__ logits, int64_t ld, const int64_t* __restrict__ labels,
    int64_t vstart, int V, int T, int rank, int tp, AuxPtrs dst, const uint32_t* epoch_ptr) {
  const int t = blockIdx.x;
  if (t >= T) return;
  const __nv_bfloat16* row = logits + static_cast<int64_t>(t) * ld;
  float m, s;
  row_stats<NT>(row, V, m, s);
  if (threadIdx.x < tp) {
    const uint32_t e = read_epoch(epoch_ptr) + 1u;
    const int64_t lab = labels[t];
    const int64_t li = lab - vstart;
    const float tgt = (lab >= 0 && li >= 0 && li < V) ? __bfloat162float(row[li]) : 0.f;
    float* st = static_cast<float*>((e & 1u) ? dst.odd[threadIdx.x] : dst.even[threadIdx.x]) +
                (static_cast<int64_t>(rank) * T + t) * 3;
    st[0] = m;
    st[1] = s;
    st[2] = tgt;
  }
}

// Same as ce_stats_scatter_kernel, but the (max, sum exp) of the row come from the LM-head
// GEMM epilogue's per-tile parts (merged by one warp per row) instead of a pass over the
// logits; only the target logit is read back.
__global__ void ce_parts_scatter_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld,
                                        const int64_t* __restrict__ labels, int64_t vstart, int V,
                                        int T, const float2* __restrict__ parts, int nparts,
                                        int rank, int tp, AuxPtrs dst, const uint32_t* epoch_ptr) {
  const int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (t >= T) return;   // warp-uniform
  const int lane = threadIdx.x & 31;
  float m = -INFINITY, sx = 0.f;
  for (int i = lane; i < nparts; i += 32) {
    const float2 q = parts[static_cast<int64_t>(t) * nparts + i];
    const float nm = fmaxf(m, q.x);
    if (nm != -INFINITY)
      sx = (m == -INFINITY ? 0.f : sx * ex2_aux((m - nm) * kLog2eAux)) +
           (q.x == -INFINITY ? 0.f : q.y * ex2_aux((q.x - nm) * kLog2eAux));
    m = nm;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, sx, o);
    const float nm = fmaxf(m, om);
    if (nm != -INFINITY)
      sx = (m == -INFINITY ? 0.f : sx * ex2_aux((m - nm) * kLog2eAux)) +
           (om == -INFINITY ? 0.f : os * ex2_aux((om - nm) * kLog2eAux));
    m = nm;
  }
  if (lane < tp) {
    const uint32_t e = read_epoch(epoch_ptr) + 1u;
    const int64_t lab = labels[t];
    const int64_t li = lab - vstart;
    const float tgt = (lab >= 0 && li >= 0 && li < V)
                          ? __bfloat162float(logits[static_cast<int64_t>(t) * ld + li]) : 0.f;
    float* st = static_cast<float*>((e & 1u) ? dst.odd[lane] : dst.even[lane]) +
                (static_cast<int64_t>(rank) * T + t) * 3;
    st[0] = m;
    st[1] = sx;
    st[2] = tgt;
  }
}

// One block per row: wait for every rank's statistics, merge them, write the row loss and
// (optionally) overwrite the local logits with d loss_row / d logits.
template <int NT>
__global__ void __launch_bounds__(NT) ce_finish_gather_kernel(
    __nv_bfloat16* logits, int64_t ld, const int64_t* __restrict__ labels, int64_t vstart,
    int V, int T, const float* even, const float* odd, int tp, float* __restrict__ loss_row,
    int write_grad, const uint32_t* flags, const uint32_t* epoch_ptr, int* status) {
  const int t = blockIdx.x;
  if (t >= T) return;
  __shared__ int ok;
  __shared__ float s_lse;
  block_wait_flags(flags, tp, epoch_ptr, status, &ok);
  if (!ok) return;
  const float* stats = (read_epoch(epoch_ptr) & 1u) ? odd : even;
  const int64_t lab = labels[t];
  const bool valid = lab >= 0;
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int r = 0; r < tp; ++r)
      M = fmaxf(M, __ldcg(stats + (static_cast<int64_t>(r) * T + t) * 3));
    float S = 0.f, tgt = 0.f;
    for (int r = 0; r < tp; ++r) {
      const float* st = stats + (static_cast<int64_t>(r) * T + t) * 3;
      const float m = __ldcg(st);
      if (m != -INFINITY) S += __ldcg(st + 1) * ex2_aux((m - M) * kLog2eAux);
      tgt += __ldcg(st + 2);
    }
    const float lse = M + __log2f(S) * kLn2Aux;
    s_lse = lse;
    loss_row[t] = valid ? lse - tgt : 0.f;
  }
  __syncthreads();
  if (!write_grad) return;
  const float lse = s_lse;
  __nv_bfloat16* row = logits + static_cast<int64_t>(t) * ld;
  const int64_t li = lab - vstart;
  const int nvec = V / 8;
  for (int c = threadIdx.x; c < nvec; c += NT) {
    uint4* p = reinterpret_cast<uint4*>(row) + c;
    const uint4 v = *p;
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      f[2 * j] = bf16_lo(wv[j]);
      f[2 * j + 1] = bf16_hi(wv[j]);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float gv = valid ? ex2_aux((f[k] - lse) * kLog2eAux) : 0.f;
      if (valid && c * 8 + k == li) gv -= 1.f;
      f[k] = gv;
    }
    uint4 o;
    o.x = pack_bf16x2(f[0], f[1]);
    o.y = pack_bf16x2(f[2], f[3]);
    o.z = pack_bf16x2(f[4], f[5]);
    o.w = pack_bf16x2(f[6], f[7]);
    *p = o;
  }
}

static AuxPtrs aux_ptrs(const std::vector<int64_t>& even, const std::vector<int64_t>& odd) {
  TORCH_CHECK(!even.empty() && even.size() <= kAuxMaxTP && odd.size() == even.size(),
              "1..8 TP ranks");
  AuxPtrs a{};
  for (size_t r = 0; r < even.size(); ++r) {
    TORCH_CHECK(even[r] % 16 == 0 && odd[r] % 16 == 0 && even[r] != 0 && odd[r] != 0,
                "symmetric slots must be 16-byte aligned");
    a.even[r] = reinterpret_cast<void*>(even[r]);
    a.odd[r] = reinterpret_cast<void*>(odd[r]);
  }
  return a;
}

static void check_ptrs(int64_t flags, int64_t epoch) {
  TORCH_CHECK(flags % 4 == 0 && flags != 0 && epoch % 4 == 0 && epoch != 0,
              "flag / epoch pointers must be 4-byte aligned device addresses");
}

}  // namespace nmb

using namespace nmb;

void tp_embedding_scatter(at::Tensor ids, at::Tensor w, int64_t vstart, int64_t rows_per_rank,
                          std::vector<int64_t> slots_even, std::vector<int64_t> slots_odd,
                          int64_t epoch_ptr) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kLong && ids.is_contiguous());
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kBFloat16 && w.is_contiguous() &&
              w.dim() == 2 && w.size(1) % 8 == 0);
  const int T = static_cast<int>(ids.numel()), H = static_cast<int>(w.size(1));
  const AuxPtrs dst = aux_ptrs(slots_even, slots_odd);
  TORCH_CHECK(rows_per_rank > 0 && T == rows_per_rank * static_cast<int64_t>(slots_even.size()),
              "tokens must equal TP x rows per rank");
  check_ptrs(4, epoch_ptr);
  const at::cuda::CUDAGuard guard(w.device());
  const int blocks = std::max(1, std::min((T + 7) / 8, 4096));
  embedding_scatter_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), w.size(0),
      vstart, T, H, static_cast<int>(rows_per_rank), dst,
      reinterpret_cast<const uint32_t*>(epoch_ptr));
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tp_embedding_collect(int64_t slot_even, int64_t slot_odd, at::Tensor out, int64_t tp,
                          int64_t flags_ptr, int64_t epoch_ptr, at::Tensor status) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.dim() == 2 &&
              out.stride(1) == 1 && out.size(1) % 8 == 0 && out.stride(0) % 8 == 0);
  TORCH_CHECK(slot_even % 16 == 0 && slot_odd % 16 == 0 && tp >= 1 && tp <= kAuxMaxTP);
  check_ptrs(flags_ptr, epoch_ptr);
  const int R = static_cast<int>(out.size(0)), H = static_cast<int>(out.size(1));
  const at::cuda::CUDAGuard guard(out.device());
  const int64_t vecs = static_cast<int64_t>(R) * (H / 8);
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((vecs + 255) / 256,
                                                                             1184)));
  embedding_collect_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(slot_even),
      reinterpret_cast<const __nv_bfloat16*>(slot_odd),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), R, H,
      reinterpret_cast<const uint32_t*>(flags_ptr), static_cast<int>(tp),
      reinterpret_cast<const uint32_t*>(epoch_ptr), status.data_ptr<int>());
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tp_embedding_bwd_gather(at::Tensor ids, std::vector<int64_t> slots_even,
                             std::vector<int64_t> slots_odd, int64_t rows_per_rank, int64_t H,
                             at::Tensor grad, int64_t vstart, int64_t flags_ptr,
                             int64_t epoch_ptr, at::Tensor status) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kLong && ids.is_contiguous());
  TORCH_CHECK(grad.is_cuda() && grad.scalar_type() == at::kFloat && grad.is_contiguous() &&
              grad.dim() == 2 && grad.size(1) == H && H % 8 == 0);
  const AuxPtrs src = aux_ptrs(slots_even, slots_odd);
  const int T = static_cast<int>(ids.numel());
  TORCH_CHECK(T == rows_per_rank * static_cast<int64_t>(slots_even.size()));
  check_ptrs(flags_ptr, epoch_ptr);
  const at::cuda::CUDAGuard guard(grad.device());
  const int blocks = std::max(1, std::min((T + 7) / 8, 4096));
  if (deterministic_mode()) {
    const auto sorted = at::sort(ids, /*stable=*/true, 0, false);
    const at::Tensor sid = std::get<0>(sorted).contiguous(), ord = std::get<1>(sorted).contiguous();
    embedding_bwd_gather_sorted_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        sid.data_ptr<int64_t>(), ord.data_ptr<int64_t>(), src, grad.data_ptr<float>(),
        grad.size(0), vstart, T, static_cast<int>(H), static_cast<int>(rows_per_rank),
        reinterpret_cast<const uint32_t*>(flags_ptr), static_cast<int>(slots_even.size()),
        reinterpret_cast<const uint32_t*>(epoch_ptr), status.data_ptr<int>());
    NMB_LAUNCHED(1);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  embedding_bwd_gather_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), src, grad.data_ptr<float>(), grad.size(0), vstart, T,
      static_cast<int>(H), static_cast<int>(rows_per_rank),
      reinterpret_cast<const uint32_t*>(flags_ptr), static_cast<int>(slots_even.size()),
      reinterpret_cast<const uint32_t*>(epoch_ptr), status.data_ptr<int>());
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tp_ce_stats_scatter(at::Tensor logits, at::Tensor labels, int64_t vstart, int64_t rank,
                         std::vector<int64_t> slots_even, std::vector<int64_t> slots_odd,
                         int64_t epoch_ptr) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 &&
              logits.stride(1) == 1 && logits.size(1) % 8 == 0 && logits.stride(0) % 8 == 0);
  TORCH_CHECK(labels.is_cuda() && labels.scalar_type() == at::kLong && labels.is_contiguous() &&
              labels.numel() == logits.size(0));
  const AuxPtrs dst = aux_ptrs(slots_even, slots_odd);
  const int tp = static_cast<int>(slots_even.size());
  TORCH_CHECK(rank >= 0 && rank < tp);
  check_ptrs(4, epoch_ptr);
  const int T = static_cast<int>(logits.size(0)), V = static_cast<int>(logits.size(1));
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(logits.device());
  ce_stats_scatter_kernel<256><<<T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
      labels.data_ptr<int64_t>(), vstart, V, T, static_cast<int>(rank), tp, dst,
      reinterpret_cast<const uint32_t*>(epoch_ptr));
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tp_ce_parts_scatter(at::Tensor logits, at::Tensor labels, int64_t vstart, at::Tensor parts,
                         int64_t nparts, int64_t rank, std::vector<int64_t> slots_even,
                         std::vector<int64_t> slots_odd, int64_t epoch_ptr) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 &&
              logits.stride(1) == 1);
  TORCH_CHECK(labels.is_cuda() && labels.scalar_type() == at::kLong && labels.is_contiguous() &&
              labels.numel() == logits.size(0));
  TORCH_CHECK(parts.is_cuda() && parts.scalar_type() == at::kFloat && parts.is_contiguous() &&
                  parts.numel() >= logits.size(0) * nparts * 2 && nparts >= 1,
              "tp_ce_parts_scatter: parts must hold T x nparts (max, sum exp) pairs");
  const AuxPtrs dst = aux_ptrs(slots_even, slots_odd);
  const int tp = static_cast<int>(slots_even.size());
  TORCH_CHECK(rank >= 0 && rank < tp);
  check_ptrs(4, epoch_ptr);
  const int T = static_cast<int>(logits.size(0)), V = static_cast<int>(logits.size(1));
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(logits.device());
  ce_parts_scatter_kernel<<<(T + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
      labels.data_ptr<int64_t>(), vstart, V, T,
      reinterpret_cast<const float2*>(parts.data_ptr<float>()), static_cast<int>(nparts),
      static_cast<int>(rank), tp, dst, reinterpret_cast<const uint32_t*>(epoch_ptr));
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tp_ce_finish_gather(at::Tensor logits, at::Tensor labels, int64_t vstart, int64_t stats_even,
                         int64_t stats_odd, int64_t tp, at::Tensor loss_row, bool write_grad,
                         int64_t flags_ptr, int64_t epoch_ptr, at::Tensor status) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 &&
              logits.stride(1) == 1 && logits.size(1) % 8 == 0 && logits.stride(0) % 8 == 0);
  TORCH_CHECK(loss_row.is_cuda() && loss_row.scalar_type() == at::kFloat &&
              loss_row.numel() == logits.size(0));
  TORCH_CHECK(stats_even % 16 == 0 && stats_odd % 16 == 0 && tp >= 1 && tp <= kAuxMaxTP);
  check_ptrs(flags_ptr, epoch_ptr);
  const int T = static_cast<int>(logits.size(0)), V = static_cast<int>(logits.size(1));
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(logits.device());
  ce_finish_gather_kernel<256><<<T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
      labels.data_ptr<int64_t>(), vstart, V, T, reinterpret_cast<const float*>(stats_even),
      reinterpret_cast<const float*>(stats_odd), static_cast<int>(tp),
      loss_row.data_ptr<float>(), write_grad ? 1 : 0,
      reinterpret_cast<const uint32_t*>(flags_ptr), reinterpret_cast<const uint32_t*>(epoch_ptr),
      status.data_ptr<int>());
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

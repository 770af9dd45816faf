// Data-parallel gradient reduction fused with the sharded AdamW update and the bf16
// parameter all-gather, over NVLink peer memory (DDP bucket all-reduce and ZeRO-1/2
// reduce-scatter + all-gather, as one path).
//
// Every rank of the replica group keeps its flat fp32 gradient buffer and its flat bf16
// parameter buffer in IPC-exported device memory that every peer has mapped. A bucket is
// cut into equal shards, one per rank. Per step:
//
//   1. signal(GRAD)     each rank, after its backward: "my gradients are final".
//   2. replica_reduce   each rank waits (bounded) for every rank's GRAD flag, then reads
//                       its own shard of the bucket from all ranks' gradient buffers
//                       (plain peer loads over NVLink, no TMA), sums in fp32, writes the
//                       sum in place into its own buffer and emits per-block partial
//                       squared norms over the norm-counted ranges. One read of each
//                       remote byte, no staging copy, no separate norm pass.
//   3. (device scalars: the partials are summed, the clip coefficient is formed)
//   4. replica_adamw_gather  AdamW over the shard (fp32 master and moments), with the
//                       gradient scaled by clip / DP read on the device, and the updated
//                       bf16 parameters stored into EVERY rank's parameter buffer (local
//                       store + peer stores): the all-gather is the optimizer's epilogue.
//   5. signal(PARAM) + replica_wait  no rank reads parameters (next forward) or writes
//                       gradients (next backward) before every rank finished 2 and 4.
//
// Waits are bounded (1 s budget plus an iteration cap); on expiry the kernel records
// 0x401 in the status word and returns without touching the data.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace nmb {

constexpr int kReplicaMax = 8;
constexpr int kSegShared = 512;   // norm segments staged in shared memory (else global)

struct ReplicaPtrs {
  const float* grad[kReplicaMax];    // each rank's flat fp32 gradient buffer (mapped here)
  __nv_bfloat16* param[kReplicaMax]; // each rank's flat bf16 parameter buffer
};

// First segment whose end is past element e (segments: sorted [start, end) pairs).
__device__ __forceinline__ int seg_lower(const int64_t* seg, int nseg, int64_t e) {
  int lo = 0, hi = nseg;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (seg[2 * mid + 1] <= e) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ bool wait_all(const uint32_t* flags, int n, const uint32_t* epoch_ptr,
                                         int* status) {
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(epoch_ptr);
  for (int r = 0; r < n; ++r)
    if (!wait_flag(flags + r, epoch, status, kStatusReplicaFlagTimeout, nullptr)) return false;
  return true;
}

__device__ __forceinline__ void block_sum_to(float acc, float* out) {
  acc = warp_sum(acc);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) *out = v;
  }
}

// grad[self][off + e] = sum_r grad[r][off + e] for e in [0, len); partials[block] = sum of
// squares of the sums over the segments (relative to the shard start).
template <bool VEC>
__global__ void __launch_bounds__(256) replica_reduce_kernel(
    ReplicaPtrs ptrs, int n, int self, int64_t off, int64_t len, const int64_t* __restrict__ seg,
    int nseg, float* __restrict__ partials, const uint32_t* flags, const uint32_t* epoch_ptr,
    int* status) {
  __shared__ int ok;
  __shared__ int64_t sseg[2 * kSegShared];
  if (threadIdx.x == 0) ok = wait_all(flags, n, epoch_ptr, status) ? 1 : 0;
  const bool staged = nseg <= kSegShared;
  if (staged)
    for (int i = threadIdx.x; i < 2 * nseg; i += blockDim.x) sseg[i] = seg[i];
  __syncthreads();
  float acc = 0.f;
  if (ok) {
    const int64_t* sg = staged ? sseg : seg;
    float* out = const_cast<float*>(ptrs.grad[self]) + off;
    const int64_t chunks = (len + 3) >> 2;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < chunks;
         c += stride) {
      const int64_t e0 = c << 2;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (VEC && e0 + 4 <= len) {
#pragma unroll
        for (int r = 0; r < kReplicaMax; ++r) {
          if (r >= n) break;
          const float4 x = __ldcg(reinterpret_cast<const float4*>(ptrs.grad[r] + off + e0));
          v[0] += x.x; v[1] += x.y; v[2] += x.z; v[3] += x.w;
        }
        *reinterpret_cast<float4*>(out + e0) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (e0 + k >= len) break;
          for (int r = 0; r < n; ++r) v[k] += __ldcg(ptrs.grad[r] + off + e0 + k);
          out[e0 + k] = v[k];
        }
      }
      if (nseg > 0) {
        int s = seg_lower(sg, nseg, e0);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int64_t e = e0 + k;
          if (e >= len) break;
          while (s < nseg && sg[2 * s + 1] <= e) ++s;
          if (s < nseg && sg[2 * s] <= e) acc += v[k] * v[k];
        }
      }
    }
  }
  block_sum_to(acc, partials + blockIdx.x);
}

struct ReplicaAdam {
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt;
};

__device__ __forceinline__ float adam_one(float g, float& p, float& m, float& v,
                                          const ReplicaAdam& hp, float lr, float gs) {
  const float gr = g * gs;
  p *= 1.f - lr * hp.wd;
  m = hp.beta1 * m + (1.f - hp.beta1) * gr;
  v = hp.beta2 * v + (1.f - hp.beta2) * gr * gr;
  p -= (lr / hp.bc1) * m / (sqrtf(v) / hp.bc2_sqrt + hp.eps);
  return p;
}

// AdamW over this rank's shard; the updated bf16 values go to every rank's parameter
// buffer at the same offset (peer stores for the others).
template <bool VEC>
__global__ void __launch_bounds__(256) replica_adamw_gather_kernel(
    ReplicaPtrs ptrs, int n, int self, int64_t off, int64_t len, float* __restrict__ master,
    float* __restrict__ m, float* __restrict__ v, ReplicaAdam hp,
    const float* __restrict__ grad_scale, const float* __restrict__ lr_ptr) {
  const float gs = grad_scale != nullptr ? *grad_scale : 1.f;
  const float lr = lr_ptr != nullptr ? *lr_ptr : hp.lr;
  const float* g = ptrs.grad[self] + off;
  const int64_t chunks = (len + 3) >> 2;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < chunks;
       c += stride) {
    const int64_t e0 = c << 2;
    if (VEC && e0 + 4 <= len) {
      const float4 gv = *reinterpret_cast<const float4*>(g + e0);
      float4 pv = *reinterpret_cast<float4*>(master + e0);
      float4 mv = *reinterpret_cast<float4*>(m + e0);
      float4 vv = *reinterpret_cast<float4*>(v + e0);
      adam_one(gv.x, pv.x, mv.x, vv.x, hp, lr, gs);
      adam_one(gv.y, pv.y, mv.y, vv.y, hp, lr, gs);
      adam_one(gv.z, pv.z, mv.z, vv.z, hp, lr, gs);
      adam_one(gv.w, pv.w, mv.w, vv.w, hp, lr, gs);
      *reinterpret_cast<float4*>(master + e0) = pv;
      *reinterpret_cast<float4*>(m + e0) = mv;
      *reinterpret_cast<float4*>(v + e0) = vv;
      uint2 o;
      o.x = pack_bf16x2(pv.x, pv.y);
      o.y = pack_bf16x2(pv.z, pv.w);
#pragma unroll
      for (int r = 0; r < kReplicaMax; ++r) {
        if (r >= n) break;
        *reinterpret_cast<uint2*>(ptrs.param[r] + off + e0) = o;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int64_t e = e0 + k;
        if (e >= len) break;
        float pe = master[e], me = m[e], ve = v[e];
        adam_one(g[e], pe, me, ve, hp, lr, gs);
        master[e] = pe;
        m[e] = me;
        v[e] = ve;
        const __nv_bfloat16 b = __float2bfloat16_rn(pe);
        for (int r = 0; r < n; ++r) ptrs.param[r][off + e] = b;
      }
    }
  }
}

// One block: wait (bounded) until every rank's flag on this channel reached our epoch.
__global__ void replica_wait_kernel(const uint32_t* flags, int n, const uint32_t* epoch_ptr,
                                    int* status) {
  if (threadIdx.x == 0) wait_all(flags, n, epoch_ptr, status);
}

static ReplicaPtrs make_ptrs(const std::vector<int64_t>& grads,
                             const std::vector<int64_t>& params) {
  TORCH_CHECK(!grads.empty() && grads.size() <= kReplicaMax, "1..8 replica ranks");
  TORCH_CHECK(params.empty() || params.size() == grads.size());
  ReplicaPtrs p{};
  for (size_t r = 0; r < grads.size(); ++r) {
    TORCH_CHECK(grads[r] != 0 && grads[r] % 16 == 0, "gradient buffers must be 16-byte aligned");
    p.grad[r] = reinterpret_cast<const float*>(grads[r]);
    if (!params.empty()) {
      TORCH_CHECK(params[r] != 0 && params[r] % 16 == 0,
                  "parameter buffers must be 16-byte aligned");
      p.param[r] = reinterpret_cast<__nv_bfloat16*>(params[r]);
    }
  }
  return p;
}

static int replica_grid(int64_t len, int device) {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const int64_t chunks = (len + 3) / 4;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((chunks + 255) / 256,
                                                                 static_cast<int64_t>(sms) * 4)));
}

}  // namespace nmb

using namespace nmb;

// Number of per-block partials replica_reduce writes for a shard of `len` elements.
int64_t replica_reduce_blocks(int64_t len, int64_t device) {
  return replica_grid(len, static_cast<int>(device));
}

void replica_reduce(std::vector<int64_t> grad_ptrs, int64_t self, int64_t off, int64_t len,
                    at::Tensor segments, at::Tensor partials, int64_t flags_ptr,
                    int64_t epoch_ptr, at::Tensor status) {
  const ReplicaPtrs p = make_ptrs(grad_ptrs, {});
  const int n = static_cast<int>(grad_ptrs.size());
  TORCH_CHECK(self >= 0 && self < n && off >= 0 && len >= 0);
  TORCH_CHECK(segments.is_cuda() && segments.scalar_type() == at::kLong &&
              segments.is_contiguous() && segments.numel() % 2 == 0);
  TORCH_CHECK(partials.is_cuda() && partials.scalar_type() == at::kFloat &&
              partials.is_contiguous());
  TORCH_CHECK(flags_ptr % 4 == 0 && flags_ptr != 0 && epoch_ptr % 4 == 0 && epoch_ptr != 0);
  const int dev = partials.device().index();
  const int grid = replica_grid(len, dev);
  TORCH_CHECK(partials.numel() >= grid, "replica_reduce: partials too small");
  const at::cuda::CUDAGuard guard(partials.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int nseg = static_cast<int>(segments.numel() / 2);
  const bool vec = off % 4 == 0;
  auto fn = vec ? replica_reduce_kernel<true> : replica_reduce_kernel<false>;
  fn<<<grid, 256, 0, stream>>>(p, n, static_cast<int>(self), off, len,
                               segments.data_ptr<int64_t>(), nseg, partials.data_ptr<float>(),
                               reinterpret_cast<const uint32_t*>(flags_ptr),
                               reinterpret_cast<const uint32_t*>(epoch_ptr),
                               status.data_ptr<int>());
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void replica_adamw_gather(std::vector<int64_t> grad_ptrs, std::vector<int64_t> param_ptrs,
                          int64_t self, int64_t off, int64_t len, at::Tensor master,
                          at::Tensor exp_avg, at::Tensor exp_avg_sq, double lr, double beta1,
                          double beta2, double eps, double wd, int64_t step,
                          c10::optional<at::Tensor> grad_scale, c10::optional<at::Tensor> lr_t) {
  const ReplicaPtrs p = make_ptrs(grad_ptrs, param_ptrs);
  const int n = static_cast<int>(grad_ptrs.size());
  TORCH_CHECK(self >= 0 && self < n && off >= 0 && len >= 0);
  for (const at::Tensor* t : {&master, &exp_avg, &exp_avg_sq})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() &&
                    t->numel() >= len,
                "replica_adamw_gather: optimizer state must be fp32 CUDA with >= len elements");
  ReplicaAdam hp;
  hp.lr = static_cast<float>(lr);
  hp.beta1 = static_cast<float>(beta1);
  hp.beta2 = static_cast<float>(beta2);
  hp.eps = static_cast<float>(eps);
  hp.wd = static_cast<float>(wd);
  hp.bc1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  hp.bc2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  const at::cuda::CUDAGuard guard(master.device());
  const bool vec = off % 4 == 0 &&
                   reinterpret_cast<uintptr_t>(master.data_ptr()) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(exp_avg.data_ptr()) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(exp_avg_sq.data_ptr()) % 16 == 0;
  auto fn = vec ? replica_adamw_gather_kernel<true> : replica_adamw_gather_kernel<false>;
  const int grid = replica_grid(len, master.device().index());
  fn<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p, n, static_cast<int>(self), off, len, master.data_ptr<float>(),
      exp_avg.data_ptr<float>(), exp_avg_sq.data_ptr<float>(), hp,
      grad_scale.has_value() ? grad_scale->data_ptr<float>() : nullptr,
      lr_t.has_value() ? lr_t->data_ptr<float>() : nullptr);
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void replica_wait(int64_t flags_ptr, int64_t n, int64_t epoch_ptr, at::Tensor status) {
  TORCH_CHECK(n >= 1 && n <= kReplicaMax);
  TORCH_CHECK(flags_ptr % 4 == 0 && flags_ptr != 0 && epoch_ptr % 4 == 0 && epoch_ptr != 0);
  const at::cuda::CUDAGuard guard(status.device());
  replica_wait_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint32_t*>(flags_ptr), static_cast<int>(n),
      reinterpret_cast<const uint32_t*>(epoch_ptr), status.data_ptr<int>());
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Context-parallel ring transport over NVLink peer memory.
//
// Each CP rank publishes a layer's K/V block into its symmetric heap slot once per
// forward (a signal makes it visible). Every ring step's attention kernel pulls the
// next step's block straight from its owner's slot into a local double buffer (the
// PullDesc warp of the attention kernels); these helpers cover the rest:
//
//  * cp_pull: the same pull as a kernel of its own, for a ring step whose keys are all
//    causally masked (no attention kernel runs that step, the next block still has to
//    arrive).
//  * cp_push: the backward's fp32 dK/dV partial for a source rank's keys, stored into
//    that rank's return slot [this rank] with peer stores (no send / receive).
//  * cp_reduce: after every rank signalled, add the partials of the contributing
//    ranks (a bit mask, known from the causal layout) to this rank's own partial.
//
// Waits are bounded (1 s budget plus an iteration cap) and record 0x501 on expiry.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace nmb {

constexpr int kCpMax = 8;

__global__ void cp_pull_kernel(PullDesc d) { pull_slice(d, threadIdx.x, blockDim.x); }

// dst (a peer's return slot, selected by the parity of the upcoming epoch) <- src.
__global__ void cp_push_kernel(const float4* __restrict__ src, float4* even, float4* odd,
                               int64_t n4, const uint32_t* epoch_ptr) {
  const uint32_t e = *reinterpret_cast<const volatile uint32_t*>(epoch_ptr) + 1u;
  float4* dst = (e & 1u) ? odd : even;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = src[i];
}

struct CpSlots {
  const float4* even[kCpMax];
  const float4* odd[kCpMax];
};

// acc[i] += sum over set bits s of mask: slot_s[i], once every rank's flag is current.
// Waiting for every rank, not only the ranks in `mask`, is what makes each layer's
// backward a barrier: with only the contributors' flags, a rank whose keys nobody sees
// (the last rank of a causal layout) could run two layers ahead and reuse a return
// slot's parity before its owner has read it (model-checked on the host).
__global__ void cp_reduce_kernel(float4* __restrict__ acc, CpSlots slots, int n, uint32_t mask,
                                 int64_t n4, const uint32_t* flags, const uint32_t* epoch_ptr,
                                 int* status) {
  __shared__ int ok;
  __shared__ uint32_t epoch;
  if (threadIdx.x == 0) {
    epoch = *reinterpret_cast<const volatile uint32_t*>(epoch_ptr);
    int good = 1;
    for (int r = 0; r < n && good; ++r)
      good = wait_flag(flags + r, epoch, status, kStatusCpFlagTimeout, nullptr) ? 1 : 0;
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  const bool odd = epoch & 1u;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 a = acc[i];
    for (int s = 0; s < n; ++s) {
      if (!((mask >> s) & 1u)) continue;
      const float4 v = __ldcg((odd ? slots.odd[s] : slots.even[s]) + i);
      a.x += v.x;
      a.y += v.y;
      a.z += v.z;
      a.w += v.w;
    }
    acc[i] = a;
  }
}

static int cp_grid(int64_t n4, int device) {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n4 + 255) / 256, sms * 4)));
}

}  // namespace nmb

using namespace nmb;

PullDesc make_pull(int64_t src, const c10::optional<at::Tensor>& dst, int64_t flag, int64_t epoch,
                   int* status);   // attention_tc.cu

void cp_pull(int64_t src, at::Tensor dst, int64_t flag_ptr, int64_t epoch_ptr, at::Tensor status) {
  const PullDesc d = make_pull(src, dst, flag_ptr, epoch_ptr, status.data_ptr<int>());
  const at::cuda::CUDAGuard guard(dst.device());
  const int grid = cp_grid(d.vec16, dst.device().index());
  cp_pull_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(d);
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void cp_push(at::Tensor src, int64_t dst_even, int64_t dst_odd, int64_t epoch_ptr) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kFloat && src.is_contiguous() &&
              src.numel() % 4 == 0 && reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0);
  TORCH_CHECK(dst_even % 16 == 0 && dst_odd % 16 == 0 && dst_even != 0 && dst_odd != 0 &&
              epoch_ptr % 4 == 0 && epoch_ptr != 0);
  const int64_t n4 = src.numel() / 4;
  const at::cuda::CUDAGuard guard(src.device());
  cp_push_kernel<<<cp_grid(n4, src.device().index()), 256, 0,
                   at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float4*>(src.data_ptr()), reinterpret_cast<float4*>(dst_even),
      reinterpret_cast<float4*>(dst_odd), n4, reinterpret_cast<const uint32_t*>(epoch_ptr));
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void cp_reduce(at::Tensor acc, std::vector<int64_t> slots_even, std::vector<int64_t> slots_odd,
               int64_t mask, int64_t flags_ptr, int64_t epoch_ptr, at::Tensor status) {
  TORCH_CHECK(acc.is_cuda() && acc.scalar_type() == at::kFloat && acc.is_contiguous() &&
              acc.numel() % 4 == 0 && reinterpret_cast<uintptr_t>(acc.data_ptr()) % 16 == 0);
  const int n = static_cast<int>(slots_even.size());
  TORCH_CHECK(n >= 1 && n <= kCpMax && static_cast<int>(slots_odd.size()) == n);
  TORCH_CHECK(flags_ptr % 4 == 0 && flags_ptr != 0 && epoch_ptr % 4 == 0 && epoch_ptr != 0);
  CpSlots s{};
  for (int r = 0; r < n; ++r) {
    TORCH_CHECK(slots_even[r] % 16 == 0 && slots_odd[r] % 16 == 0);
    s.even[r] = reinterpret_cast<const float4*>(slots_even[r]);
    s.odd[r] = reinterpret_cast<const float4*>(slots_odd[r]);
  }
  const int64_t n4 = acc.numel() / 4;
  const at::cuda::CUDAGuard guard(acc.device());
  cp_reduce_kernel<<<cp_grid(n4, acc.device().index()), 256, 0,
                     at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<float4*>(acc.data_ptr()), s, n, static_cast<uint32_t>(mask), n4,
      reinterpret_cast<const uint32_t*>(flags_ptr), reinterpret_cast<const uint32_t*>(epoch_ptr),
      status.data_ptr<int>());
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

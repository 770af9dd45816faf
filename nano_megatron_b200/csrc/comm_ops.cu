// Symmetric memory over NVLink for the fused tensor-parallel collectives.
//
// Every TP rank allocates one device buffer, exports a CUDA IPC handle, and maps
// every peer's buffer into its own address space (handles travel over the c10d
// store as bytes). Inside a buffer: a flag array (one 32-bit slot per source
// rank and channel) followed by data regions the Python layer carves out.
//
// Synchronisation is by monotonically increasing epochs, one device-resident counter
// per channel and rank. The signal kernel advances the counter and, after this rank's
// stores, writes the new epoch with a system-scope release store into slot [its rank]
// of every rank's flag array (itself included); a consumer reads the counter and waits
// (bounded, 1 s budget) until the slots reach it, with acquire loads. Keeping the epoch
// on the device means no launch carries a per-call value, so a sequence of fused
// collectives can be captured once in a CUDA graph and replayed. The waits never spin
// forever: on timeout they record an error in the status word and the kernel returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <string>

#include "common.cuh"

namespace nmb {

constexpr int kCommMaxTP = 8;

struct FlagTargets {
  uint32_t* flag[kCommMaxTP];  // destination flag slot (already offset to [channel][my rank])
};

__global__ void peer_signal_kernel(FlagTargets t, int n, uint32_t* epoch_ptr) {
  __shared__ uint32_t e;
  if (threadIdx.x == 0) {
    e = *epoch_ptr + 1u;
    *epoch_ptr = e;
  }
  __syncthreads();
  const int r = threadIdx.x;
  if (r < n) {
    fence_sc_sys();  // this rank's earlier stores (previous kernels included) before the flag
    st_release_sys(t.flag[r], e);
  }
}

// Copy this rank's [rows, cols] shard into its symmetric slot of the upcoming epoch's
// parity (*epoch_ptr + 1); the signal kernel that follows publishes it.
__global__ void ag_publish_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int64_t rows,
                                  int64_t cols, __nv_bfloat16* even, __nv_bfloat16* odd,
                                  const uint32_t* epoch_ptr) {
  const uint32_t e = *reinterpret_cast<const volatile uint32_t*>(epoch_ptr) + 1u;
  __nv_bfloat16* dst = (e & 1u) ? odd : even;
  const int64_t vec = cols / 8, total = rows * vec;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vec, c = (i - r * vec) * 8;
    *reinterpret_cast<uint4*>(dst + r * cols + c) =
        *reinterpret_cast<const uint4*>(x + r * ldx + c);
  }
}

// out[i, :] = sum_r staging[r][i, :] (+ residual[i, :]); waits for every rank's epoch first.
__global__ void rs_reduce_kernel(const __nv_bfloat16* even, const __nv_bfloat16* odd, int tp,
                                 int64_t rows, int64_t n, __nv_bfloat16* __restrict__ out,
                                 int64_t ldo, const __nv_bfloat16* __restrict__ res, int64_t ldr,
                                 const uint32_t* flags, const uint32_t* epoch_ptr, int* status) {
  __shared__ int ok;
  __shared__ uint32_t epoch;
  if (threadIdx.x == 0) {
    epoch = *reinterpret_cast<const volatile uint32_t*>(epoch_ptr);
    int good = 1;
    for (int r = 0; r < tp && good; ++r)
      good = wait_flag(flags + r, epoch, status, kStatusPeerFlagTimeout,
                       reinterpret_cast<volatile int*>(status));
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  const __nv_bfloat16* __restrict__ staging = (epoch & 1u) ? odd : even;
  const int64_t vec_per_row = n / 8;  // 8 bf16 = 16 bytes
  const int64_t total = rows * vec_per_row;
  const int64_t slot = rows * n;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / vec_per_row, c8 = (i - row * vec_per_row) * 8;
    float acc[8];
    if (res != nullptr) {
      const uint4 rv = *reinterpret_cast<const uint4*>(res + row * ldr + c8);
      const uint32_t w[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = bf16_lo(w[j]);
        acc[2 * j + 1] = bf16_hi(w[j]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    }
    for (int r = 0; r < tp; ++r) {
      const uint4 sv = *reinterpret_cast<const uint4*>(staging + r * slot + row * n + c8);
      const uint32_t w[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] += bf16_lo(w[j]);
        acc[2 * j + 1] += bf16_hi(w[j]);
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + row * ldo + c8) = o;
  }
}

}  // namespace nmb

using namespace nmb;

// Allocate `bytes` of zeroed device memory for symmetric use. Returns the buffer as a
// uint8 tensor (freed with cudaFree when the tensor dies) and its IPC handle bytes.
std::tuple<at::Tensor, py::bytes> symm_alloc(int64_t bytes, int64_t device) {
  TORCH_CHECK(bytes > 0);
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&ptr, static_cast<size_t>(bytes)));
  C10_CUDA_CHECK(cudaMemset(ptr, 0, static_cast<size_t>(bytes)));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, ptr));
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device);
  at::Tensor t = at::from_blob(ptr, {bytes}, [](void* p) { cudaFree(p); }, opts);
  return {t, py::bytes(reinterpret_cast<const char*>(&h), sizeof(h))};
}

int64_t symm_open(py::bytes handle, int64_t device) {
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(ptr);
}

void symm_close(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

// Advance the channel's device epoch and write it into every flag slot address in
// `targets` (one per destination rank).
void peer_signal(std::vector<int64_t> targets, int64_t epoch_ptr) {
  const int n = static_cast<int>(targets.size());
  TORCH_CHECK(n >= 1 && n <= kCommMaxTP);
  FlagTargets t{};
  for (int r = 0; r < n; ++r) {
    TORCH_CHECK(targets[r] % 4 == 0);
    t.flag[r] = reinterpret_cast<uint32_t*>(targets[r]);
  }
  TORCH_CHECK(epoch_ptr % 4 == 0 && epoch_ptr != 0);
  peer_signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      t, n, reinterpret_cast<uint32_t*>(epoch_ptr));
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ag_publish(at::Tensor x, int64_t even_ptr, int64_t odd_ptr, int64_t epoch_ptr) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 &&
              x.stride(1) == 1 && x.size(1) % 8 == 0 && x.stride(0) % 8 == 0);
  TORCH_CHECK(even_ptr % 16 == 0 && odd_ptr % 16 == 0 && epoch_ptr % 4 == 0 && epoch_ptr != 0);
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t vecs = x.size(0) * (x.size(1) / 8);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((vecs + 255) / 256, 1184)));
  ag_publish_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), x.size(0), x.size(1),
      reinterpret_cast<__nv_bfloat16*>(even_ptr), reinterpret_cast<__nv_bfloat16*>(odd_ptr),
      reinterpret_cast<const uint32_t*>(epoch_ptr));
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rs_reduce(int64_t staging_even, int64_t staging_odd, int64_t tp, at::Tensor out,
               c10::optional<at::Tensor> residual, int64_t flags_ptr, int64_t epoch_ptr,
               at::Tensor status) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.dim() == 2 &&
              out.stride(1) == 1);
  const int64_t rows = out.size(0), n = out.size(1);
  TORCH_CHECK(n % 8 == 0 && out.stride(0) % 8 == 0 && staging_even % 16 == 0 &&
              staging_odd % 16 == 0 && epoch_ptr % 4 == 0 && epoch_ptr != 0);
  const __nv_bfloat16* res = nullptr;
  int64_t ldr = 0;
  if (residual.has_value()) {
    TORCH_CHECK(residual->scalar_type() == at::kBFloat16 && residual->stride(1) == 1 &&
                residual->size(0) == rows && residual->size(1) == n &&
                residual->stride(0) % 8 == 0);
    res = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    ldr = residual->stride(0);
  }
  const at::cuda::CUDAGuard guard(out.device());
  const int64_t vecs = rows * (n / 8);
  int dev_sms = 0;
  cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, out.device().index());
  const int block = 256;
  const int grid = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>((vecs + block - 1) / block, static_cast<int64_t>(dev_sms) * 4)));
  rs_reduce_kernel<<<grid, block, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(staging_even),
      reinterpret_cast<const __nv_bfloat16*>(staging_odd), static_cast<int>(tp), rows, n,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), res, ldr,
      reinterpret_cast<const uint32_t*>(flags_ptr), reinterpret_cast<const uint32_t*>(epoch_ptr),
      status.data_ptr<int>());
  NMB_LAUNCHED(1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

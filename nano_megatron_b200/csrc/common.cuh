// Shared device helpers for the sm_100a kernels of nano_megatron_b200.
//
// Everything here is inline PTX for Blackwell (sm_100a): mbarriers, TMA tensor
// loads, tcgen05 tensor-core/TMEM instructions, and a bounded-wait discipline.
// No wait in any kernel of this library spins forever: every wait carries a
// wall-clock budget (%globaltimer) and, when it runs out, records an error code
// in a device status word that the host reads after the step, then returns
// false so the caller can unwind without hanging the GPU.
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "launch_counter.h"

namespace nmb {


// Make the device's primary context current on the calling host thread.
// Driver-API calls such as cuTensorMapEncodeTiled crash in a thread that has no
// current context yet (e.g. an autograd worker whose first CUDA call is ours,
// since device guards skip cudaSetDevice when the index already matches).
// The driver entry point is resolved through the runtime, so the library does not link
// against libcuda and imports on machines without a GPU driver.
inline void ensure_current_context(int device) {
  using GetCurrentFn = CUresult (*)(CUcontext*);
  static const GetCurrentFn get_current = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return reinterpret_cast<GetCurrentFn>(fn);
  }();
  CUcontext ctx = nullptr;
  if (get_current == nullptr || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr)
    cudaSetDevice(device);
}

// ---------------------------------------------------------------- status word
// Error codes written into the device status word (first writer wins).
enum StatusCode : int {
  kStatusOk = 0,
  kStatusGemmProducerTimeout = 0x101,
  kStatusGemmMmaTimeout = 0x102,
  kStatusGemmEpilogueTimeout = 0x103,
  kStatusAttnTimeout = 0x201,
  kStatusPeerFlagTimeout = 0x301,
  kStatusPeerBarrierTimeout = 0x302,
  kStatusReplicaFlagTimeout = 0x401,
  kStatusCpFlagTimeout = 0x501,
};

// Wall-clock budget for any single wait, in nanoseconds (2 s). Pipeline waits
// inside one kernel finish in microseconds; this only trips on a real fault.
constexpr unsigned long long kWaitBudgetNs = 2000000000ull;
// Budget for waits on another GPU's flag (1 s): shorter than the in-kernel pipeline
// waits, so when a peer is missing the peer wait is the one that reports.
constexpr unsigned long long kPeerWaitBudgetNs = 1000000000ull;
// Iteration caps: a second, clock-independent bound on every spin loop. Each is well
// above what the wall-clock budget allows (a try_wait or an NVLink load takes tens of ns
// or more per round), so in practice the time budget trips first.
constexpr uint32_t kMbarMaxIters = 1u << 28;
constexpr uint32_t kPeerMaxIters = 1u << 25;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

// ------------------------------------------------------------------- basics
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ----------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait on an mbarrier phase. Returns false (after recording `code`)
// when the budget runs out or when another role of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code,
                                          volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long start = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0u) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (globaltimer_ns() - start > kWaitBudgetNs || it >= kMbarMaxIters) {
        record_status(status, code);
        if (abort_flag != nullptr) *abort_flag = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}

// 2-D tiled TMA load (no multicast): box lands at `smem_dst`, completion is
// signalled on `bar` as transaction bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* desc, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 2-D tiled TMA store of a swizzled smem tile to global memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const void* desc, const void* smem_src, int32_t x,
                                             int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(desc)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_store_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until every committed bulk store has finished *reading* its shared-memory source.
// Wait until every committed bulk store of this thread has been performed (written).
__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Order generic-proxy writes (e.g. a peer's stores observed through an acquire) before
// subsequent async-proxy (TMA) reads of global memory by this thread.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ------------------------------------------------------------ peer flags (NVLink)
// A flag word lives in a rank's symmetric buffer; peers write it with a system-scope
// release store after their data stores, the owner polls it with acquire loads.
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_sc_sys() { asm volatile("fence.sc.sys;" ::: "memory"); }

// Device-scope flag pair (producer and consumer on this GPU, e.g. two CTAs of one kernel).
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until *flag has reached `epoch` (wrap-safe compare). Returns false after
// recording `code` when the budget runs out or another role aborted.
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t epoch, int* status,
                                          int code, volatile int* abort_flag) {
  if (static_cast<int32_t>(ld_acquire_sys(flag) - epoch) >= 0) return true;
  const unsigned long long start = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (static_cast<int32_t>(ld_acquire_sys(flag) - epoch) >= 0) return true;
    if ((it & 63u) == 0u) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (globaltimer_ns() - start > kPeerWaitBudgetNs || it >= kPeerMaxIters) {
        record_status(status, code);
        if (abort_flag != nullptr) *abort_flag = 1;
        return false;
      }
    }
    __nanosleep(64);
  }
}

// ------------------------------------------------------------ ring pull (peer -> local)
// A kernel computing on block i of a ring can bring block i+1 into local memory while it
// runs: each CTA copies its slice of `vec16` 16-byte words from `src` (another GPU's
// memory, mapped here) to `dst` (this GPU) with plain loads and stores, after a bounded
// wait until the owner's publish flag reaches the expected epoch. The next kernel on the
// stream reads `dst` (kernel boundary = ordering); the TMA loads of that kernel therefore
// read only this GPU's memory.
struct PullDesc {
  const uint4* src;            // nullptr: nothing to pull
  uint4* dst;
  long long vec16;
  const uint32_t* flag;        // owner's publish flag (a slot in this rank's flag array)
  const uint32_t* epoch_ptr;   // device counter holding the epoch to wait for
  int* status;
};

__device__ __forceinline__ void pull_slice(const PullDesc& d, int tid, int nthreads) {
  if (d.src == nullptr) return;
  const uint32_t e = *reinterpret_cast<const volatile uint32_t*>(d.epoch_ptr);
  if (!wait_flag(d.flag, e, d.status, kStatusCpFlagTimeout, nullptr)) return;
  const long long ncta = static_cast<long long>(gridDim.x) * gridDim.y * gridDim.z;
  const long long cta =
      blockIdx.x + static_cast<long long>(gridDim.x) * (blockIdx.y + static_cast<long long>(
                                                                         gridDim.y) * blockIdx.z);
  const long long per = (d.vec16 + ncta - 1) / ncta;
  const long long lo = cta * per;
  const long long hi = lo + per < d.vec16 ? lo + per : d.vec16;
  for (long long i = lo + tid; i < hi; i += nthreads) d.dst[i] = __ldcg(d.src + i);
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16/f16 inputs, fp32 accumulate.
__device__ __forceinline__ void umma_f16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T (A operand read from tensor memory).
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives the
// 32 columns of TMEM lane (lane_base + i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// --------------------------------------------------- UMMA shared-memory descriptors
// Blackwell shared-memory matrix descriptor for a 128-byte-swizzled tile
// (layout type 2), descriptor version 1, base offset 0 (tiles are 1024-B aligned).
// Fields (16-byte units): start address [0,14), leading byte offset [16,30),
// stride byte offset [32,46); version at bit 46; layout type at [61,64).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
// a_mn / b_mn select MN-major (transposed) operands.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4)                                  // D format: f32
         | (1u << 7)                                // A format: bf16
         | (1u << 10)                               // B format: bf16
         | ((a_mn ? 1u : 0u) << 15)                 // A major
         | ((b_mn ? 1u : 0u) << 16)                 // B major
         | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

// ------------------------------------------------------------ small math
__device__ __forceinline__ float bf16_lo(uint32_t v) {
  return __uint_as_float(v << 16);
}
__device__ __forceinline__ float bf16_hi(uint32_t v) {
  return __uint_as_float(v & 0xFFFF0000u);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}


// ------------------------------------------------------- deterministic mode
// Process-wide switch (default off). When on, every kernel of this library that would
// sum fp32 partials with atomics, in an order the hardware schedule decides, sums them in
// a fixed order instead: split-K weight gradients run unsplit, the attention backward
// stores one dQ partial per key block and sums the blocks in order, and the RMSNorm
// weight gradient and the embedding backward reduce rows in row / token order. Runs are
// then bitwise reproducible for a fixed launch configuration. Defined in fused_ops.cu.
bool deterministic_mode();

// Deterministic scatter-add of bf16 rows into fp32 `grad` rows ([V, H], H % 8 == 0,
// 16-byte aligned). `sorted_ids` holds the T token ids sorted stably and `order` their
// token indices, so equal ids form runs in token order. One warp per run adds the run's
// rows, in that order, to the run's grad row with plain loads and stores: no two warps
// touch the same row, so the result does not depend on the schedule. Ids outside
// [vstart, vstart + V) are skipped. `chunk_of(t, c)` returns the c-th 16-byte chunk
// (8 bf16) of token t's row.
template <class ChunkOf>
__device__ __forceinline__ void add_sorted_runs(const int64_t* __restrict__ sorted_ids,
                                                const int64_t* __restrict__ order, int T,
                                                int64_t vstart, int64_t V, int H,
                                                float* __restrict__ grad, ChunkOf chunk_of) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x / 32;
  const int nvec = H / 8;
  for (int p = blockIdx.x * warps + threadIdx.x / 32; p < T; p += gridDim.x * warps) {
    const int64_t id = sorted_ids[p];
    if (p > 0 && sorted_ids[p - 1] == id) continue;  // not the first token of its run
    const int64_t local = id - vstart;
    if (local < 0 || local >= V) continue;
    int end = p + 1;
    while (end < T && sorted_ids[end] == id) ++end;
    float4* dst = reinterpret_cast<float4*>(grad + local * H);
    for (int c = lane; c < nvec; c += 32) {
      float4 a = dst[2 * c], b = dst[2 * c + 1];
      for (int j = p; j < end; ++j) {
        const uint4 v = chunk_of(order[j], c);
        a.x += bf16_lo(v.x);
        a.y += bf16_hi(v.x);
        a.z += bf16_lo(v.y);
        a.w += bf16_hi(v.y);
        b.x += bf16_lo(v.z);
        b.y += bf16_hi(v.z);
        b.z += bf16_lo(v.w);
        b.w += bf16_hi(v.w);
      }
      dst[2 * c] = a;
      dst[2 * c + 1] = b;
    }
  }
}

}  // namespace nmb

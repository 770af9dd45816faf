// Allocation-free entry point of the flash-attention backward.
//
// This entry point has no counterpart in the reference implementation; it is an
// addition of this library for callers that must not allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is not allowed or not wanted,
// for example a caller executing inside a custom memory allocator's own
// callbacks (re-entering the allocator would deadlock), a serving or
// real-time runtime that reserved all device memory up front and forbids any
// later allocation, or a host program without PyTorch that links this shared
// library directly and owns every buffer itself. Such a caller passes its own
// inputs and outputs; the two temporary buffers the backward needs (per-row
// softmax statistics and the fp32 dQ accumulator) come from a fixed array that
// lives in the library's own device memory instead of from an allocator.
//
// Limits and rules:
//  * Scratch capacity is NMB_NOALLOC_SCRATCH_FLOATS floats (32 MiB) per GPU,
//    reserved on every GPU that loads the library until the process exits.
//    A call needs B*Hq*Sq*(D+1) floats (plus up to 64 floats of alignment);
//    larger problems are rejected with NMB_NOALLOC_TOO_LARGE.
//  * The first call on a device (made with that device current) looks up the
//    scratch address with cudaGetSymbolAddress; make that first call before any
//    CUDA stream capture.
//  * All calls share the one scratch array: calls that can overlap on the GPU
//    (different streams without ordering) race and corrupt each other. The
//    kernels clear the parts that must start at zero on every call.
//  * seq_k == 0 (no keys) is valid: dq is written as zeros and dk/dv are empty.
//  * A CUDA error that an earlier, unrelated call left pending is cleared before the
//    launches (cudaGetLastError), so NMB_NOALLOC_LAUNCH_FAILED reports only a failure
//    of this call's own kernel launches.
//  * Layout: q/o/dout/dq are contiguous [B, Sq, Hq, D]; k/v/dk/dv contiguous
//    [B, Sk, Hkv, D]; lse is [B, Hq, Sq] fp32 (base-2 log-sum-exp from the
//    forward); bf16 tensors, D = 64 or 128, Hq a multiple of Hkv.
#pragma once

#include <cuda_runtime.h>

#define NMB_NOALLOC_SCRATCH_FLOATS (8ll * 1024 * 1024)

enum {
  NMB_NOALLOC_OK = 0,
  NMB_NOALLOC_BAD_ARGUMENT = 1,
  NMB_NOALLOC_TOO_LARGE = 2,
  NMB_NOALLOC_SETUP_FAILED = 3,
  NMB_NOALLOC_LAUNCH_FAILED = 4,
};

#ifdef __cplusplus
extern "C" {
#endif

// Returns NMB_NOALLOC_OK or one of the error codes above; allocates nothing.
__attribute__((visibility("default"))) int nmb_flash_attn_bwd_noalloc(
    const void* q, const void* k, const void* v, const void* o, const void* dout,
    const float* lse, void* dq, void* dk, void* dv, int batch, int seq_q, int seq_k,
    int heads_q, int heads_kv, int head_dim, float softmax_scale, int causal, int q_offset,
    int k_offset, cudaStream_t stream);

// Human-readable text for a return code of nmb_flash_attn_bwd_noalloc.
__attribute__((visibility("default"))) const char* nmb_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif

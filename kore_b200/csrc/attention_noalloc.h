// Allocation-free attention backward: a C entry point for callers that cannot
// allocate GPU memory. It has no counterpart in the reference.
//
// Who needs it: code that must not call cudaMalloc (or any allocating library
// routine) while it runs, for example a caller that has handed all device
// memory to its own pool or arena, a runtime in which allocation is forbidden
// after start-up, or a plain C/C++ host program that does not link PyTorch's
// caching allocator. The regular entry point (kore::attn_bwd) needs two
// scratch tensors supplied by its caller; this variant keeps that scratch in a
// fixed array inside the library instead.
//
// Scratch: one file-scope device array of KORE_ATTN_NOALLOC_SCRATCH_BYTES
// (64 MiB) on every GPU that loads the library, held until the process exits.
// It holds the fp32 dQ accumulator (T*Hq*128 floats) and the per-row delta
// (T*Hq floats), so a call needs T * Hq * 129 * 4 <= 64 MiB, i.e.
// T * Hq <= 130,055 (for example 2048 tokens x 40 heads). Larger calls are
// rejected with KORE_NOALLOC_ERR_TOO_LARGE before anything is launched.
//
// Set-up: the first call on each device looks up the array's device address
// (cudaGetSymbolAddress) with that device current; make that first call
// before any stream capture. Every call on a device shares the one array, and
// the kernels zero what must start at zero: calls that overlap on the GPU
// (different streams, no ordering between them) race on it.
//
// Layouts (bf16, head_dim 128): dout/q/dq [T, Hq, 128] and k/v/dk/dv
// [T, Hkv, 128], heads contiguous, each with a row stride (elements between
// tokens) that is a multiple of 8, at least the row width (Hq*128 or
// Hkv*128) and below 2^31; o [T, Hq, 128] contiguous; these eight pointers
// must be 16-byte aligned. lse [Hq, T] fp32 (natural log, as written by the
// forward) and cu_seqlens int32 [nseq+1] on the device need 4-byte alignment.
// max_seqlen must not exceed T. dq/dk/dv rows are written in place: columns
// between one row's end and the next row's start are left untouched.
//
// Return value: 0 means the arguments were valid and the kernels were
// launched on `stream`, not that they finished. The kernels' waits are
// bounded; if one gives up, the outputs are incomplete and the kernels record
// an error that kore_attn_noalloc_read_error() returns (and clears) after
// synchronizing the device.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#define KORE_ATTN_NOALLOC_SCRATCH_BYTES (64u << 20)

enum {
  KORE_NOALLOC_OK = 0,
  KORE_NOALLOC_ERR_TOO_LARGE = 1,   // T * Hq * 129 * 4 bytes exceed the scratch array
  KORE_NOALLOC_ERR_ARGS = 2,        // bad shape, stride or alignment
  KORE_NOALLOC_ERR_SETUP = 3,       // device query / symbol address lookup failed
  KORE_NOALLOC_ERR_LAUNCH = 4,      // a kernel launch failed
};

extern "C" __attribute__((visibility("default"))) int kore_attn_bwd_noalloc(
    const void* dout, int64_t ld_dout, const void* q, int64_t ld_q, const void* k, int64_t ld_k,
    const void* v, int64_t ld_v, const void* o, const float* lse, const int* cu_seqlens,
    int nseq, int max_seqlen, int T, int Hq, int Hkv, float scale, void* dq, int64_t ld_dq,
    void* dk, int64_t ld_dk, void* dv, int64_t ld_dv, cudaStream_t stream);

// 0 = no kernel error since the last read, 1 = a bounded wait timed out,
// -1 = the device could not be queried. Synchronizes the current device.
extern "C" __attribute__((visibility("default"))) int kore_attn_noalloc_read_error(void);

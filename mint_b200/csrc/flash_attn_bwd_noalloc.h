// Allocation-free FlashAttention backward: a C entry point for host code that cannot allocate
// device memory. This entry point has no counterpart in the reference framework.
//
// Who needs it: callers that are not allowed to call cudaMalloc / cudaFree (or an allocator built
// on them) at the point where they run the backward pass -- for example a runtime that pre-plans
// every device buffer and forbids allocation while it executes, a plugin hosted inside another
// framework's memory pool, or C code that links the library without PyTorch's caching allocator.
// The regular `mint_b200._C.flash_attn_bwd` allocates its outputs and two work buffers (an fp32
// dQ accumulator and the per-row delta = rowsum(dO * O)) with ATen on every call; here the caller
// passes the outputs and the work buffers come from one fixed array compiled into the library.
//
// Scratch: a file-scope `__device__` array of about 16.1 MiB (an fp32 dQ accumulator for up to
// B * T * Hq = 32768 query rows of head_dim 128, the matching delta rows and a spare status word).
// Every GPU on which the library is loaded keeps this array until the process exits. Calls with
// B * T * Hq above 32768 are rejected with an error (return value 2) and launch nothing.
//
// Set-up: the first call on a device (with that device current) looks up the array's device
// address with cudaGetSymbolAddress and raises the main kernel's shared-memory limit; make that
// first call before any CUDA stream capture. Later calls on that device only enqueue work.
//
// Sharing: every call on a device uses the same array, and the array keeps the last call's
// contents. Each call clears the dQ accumulator (cudaMemsetAsync on `stream`) before its kernels.
// Calls that can overlap on the GPU -- on different streams without ordering between them, or
// from several host threads -- race on the array and give wrong gradients; order them on one
// stream or synchronize between them.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

// Gradients of softmax(scale * Q K^T + mask) V with respect to Q, K and V (bf16, head_dim 128,
// grouped-query attention with Hq a multiple of Hkv). Layouts are contiguous row-major:
//   q, dout, o, dq : [B, T, Hq, 128] bf16       k, v, dk, dv : [B, T, Hkv, 128] bf16
//   lse            : [B, Hq, T] fp32 natural-log softmax normalizer saved by the forward pass
//   doc            : [B, T] int32 document ids (attention stays inside a document), or NULL
// causal != 0 keeps keys j <= i; window >= 0 also drops keys with i - j > window (< 0: no window).
// `status` is an optional device pointer to a 32-bit word: when a kernel gives up on a bounded wait
// (4 s) the call ORs an error bit into it (a one-thread kernel after the backward kernels moves the
// bits there), and the gradients of that call must not be used. With NULL the bits stay in a word
// inside the library's array; read and clear them with mint_flash_attn_bwd_noalloc_status.
// `doc`: with document ids the kernels compare ids element by element and skip no key tiles (the
// regular binding also passes precomputed document bounds and skips whole tiles outside a query's
// document), so packed documents are correct here but slower than through the binding.
// All work is enqueued on `stream`; the call returns before the GPU finishes.
// Returns 0 on success, 1 for a bad argument, 2 for a size above the scratch limit, 3 for a CUDA
// error during set-up or launch. On failure a message is written to `err` (if non-NULL,
// truncated to `err_len` bytes including the terminating zero).
int mint_flash_attn_bwd_noalloc(const void* dout, const void* q, const void* k, const void* v, const void* o,
                                const float* lse, const int* doc, void* dq, void* dk, void* dv, int B, int T,
                                int Hq, int Hkv, int causal, int window, float scale, unsigned int* status,
                                cudaStream_t stream, char* err, size_t err_len);

// Reads (and with reset != 0 clears) the internal status word of the current device: the error
// bits of every call made with status == NULL. Synchronizes the device first, so it is a host-side
// check between steps, not something to call inside a stream capture. Returns 0 on success.
int mint_flash_attn_bwd_noalloc_status(int reset, unsigned int* out);

// Largest B * T * Hq that mint_flash_attn_bwd_noalloc accepts.
#define MINT_FLASH_ATTN_BWD_NOALLOC_MAX_ROWS 32768

#ifdef __cplusplus
}
#endif

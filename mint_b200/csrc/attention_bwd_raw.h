// Raw-pointer interface to the FlashAttention backward kernels of attention_bwd_sm100.cu, for
// host code that owns every device buffer itself (no ATen allocation on this path).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace mint {

struct FlashBwdRaw {
  const void* dout;  // [B, T, Hq, 128] bf16
  const void* q;     // [B, T, Hq, 128] bf16
  const void* k;     // [B, T, Hkv, 128] bf16
  const void* v;     // [B, T, Hkv, 128] bf16
  const void* o;     // [B, T, Hq, 128] bf16 (forward output)
  const float* lse;  // [B, Hq, T] natural-log softmax normalizer from the forward
  const int* doc;    // [B, T] document ids, or null
  void* dq;          // [B, T, Hq, 128] bf16 out
  void* dk;          // [B, T, Hkv, 128] bf16 out
  void* dv;          // [B, T, Hkv, 128] bf16 out
  float* dq_acc;     // [B, T, Hq, 128] fp32 work buffer, zero on entry
  float* delta;      // [B, Hq, T] fp32 work buffer
  uint32_t* status;  // device status word (error bits ORed in by timed-out waits)
  int B, T, Hq, Hkv;
  bool causal;
  int window;  // keys with i - j > window are masked; < 0 disables the window
  float scale;
};

// Enqueues the delta, main and dQ-cast kernels on `stream`. Throws c10::Error on a launch error.
void flash_attn_bwd_launch_raw(const FlashBwdRaw& a, cudaStream_t stream);

// Dynamic shared memory of the main backward kernel, in bytes.
int flash_attn_bwd_smem_bytes();

// Raises the main kernel's dynamic shared-memory limit on the current device (once per device).
void flash_attn_bwd_configure_current_device();

}  // namespace mint

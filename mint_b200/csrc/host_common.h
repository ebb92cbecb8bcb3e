// Host-side helpers shared by the extension's translation units: per-device status word,
// TMA tensor-map encoding through the driver entry point (no link against libcuda), and
// argument checks.
#pragma once

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstdint>

namespace mint {

#define MINT_CHECK(cond, ...) TORCH_CHECK(cond, "mint_b200: ", __VA_ARGS__)
#define MINT_CUDA_CHECK(expr)                                                                       \
  do {                                                                                              \
    cudaError_t err__ = (expr);                                                                     \
    TORCH_CHECK(err__ == cudaSuccess, "mint_b200 CUDA error: ", cudaGetErrorString(err__), " at ", \
                __FILE__, ":", __LINE__);                                                           \
  } while (0)

// Device pointer to this device's status block (allocated once per device): word 0 is the status
// word (zero = no kernel reported an error), bytes 8..15 the wait limit in ns of every bounded spin.
constexpr uint64_t kDefaultWaitLimitNsHost = 4000000000ull;
uint32_t* status_ptr(int device);
uint32_t read_status_word(int device, bool reset);
void set_wait_limit_ns(int device, uint64_t ns);
uint64_t wait_limit_ns(int device);

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with row stride `ld` elements,
// box = [box_rows, box_cols], 128-byte swizzle. Requires cols*2 and ld*2 to be multiples of 16.
CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                              uint32_t box_cols, bool swizzle128);

// 3-D bf16 tensor map: dims (innermost first) {d0, d1, d2}, strides in elements for d1, d2.
CUtensorMap make_tmap_3d_bf16(const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                              uint64_t stride2, uint32_t box0, uint32_t box1, uint32_t box2, bool swizzle128);

// 2-D tensor map of any dtype (element size `esize` bytes, CUtensorMapDataType `dtype`),
// row-major [rows, cols] with row stride `ld` elements; `swizzle` is a CUtensorMapSwizzle value.
CUtensorMap make_tmap_2d(const void* base, int dtype, int esize, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint32_t box_rows, uint32_t box_cols, int swizzle);

// 3-D tensor map of any dtype: dims (innermost first) {d0, d1, d2}, strides in elements for d1, d2.
CUtensorMap make_tmap_3d(const void* base, int dtype, int esize, uint64_t d0, uint64_t d1, uint64_t d2,
                         uint64_t stride1, uint64_t stride2, uint32_t box0, uint32_t box1, uint32_t box2, int swizzle);

// 4-D tensor map of any dtype: dims (innermost first), strides in elements for dims 1..3.
CUtensorMap make_tmap_4d(const void* base, int dtype, int esize, const uint64_t (&dims)[4], const uint64_t (&strides)[3],
                         const uint32_t (&box)[4], int swizzle);

int num_sms(int device);

// Raise a clear error when a kernel's dynamic shared memory exceeds the device's per-block opt-in
// limit. Call before cudaFuncSetAttribute(MaxDynamicSharedMemorySize): on this driver an
// over-limit request crashed the process instead of returning an error code.
void check_smem_optin(int bytes, int device, const char* kernel);

// Number of kernels launched by this extension since process start (bench.py's gpu_launches).
void count_launch(int n = 1);
int64_t launch_count();

inline void check_cuda(const at::Tensor& t, const char* name) {
  MINT_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

inline void check_contig(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  MINT_CHECK(t.is_contiguous(), name, " must be contiguous");
}

}  // namespace mint

// Host helpers: status words, tensor-map encoding, SM counts.
#include "host_common.h"

#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>
#include <vector>

namespace mint {

namespace {
std::atomic<int64_t> g_launches{0};
std::mutex g_mu;
std::vector<uint32_t*> g_status(64, nullptr);
std::vector<int> g_sms(64, 0);

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  MINT_CHECK(fn != nullptr, "cuTensorMapEncodeTiled entry point unavailable");
  return fn;
}
}  // namespace

void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
int64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }

uint32_t* status_ptr(int device) {
  std::lock_guard<std::mutex> lk(g_mu);
  MINT_CHECK(device >= 0 && device < 64, "bad device index");
  if (g_status[device] == nullptr) {
    void* p = nullptr;
    MINT_CUDA_CHECK(cudaMalloc(&p, 256));
    MINT_CUDA_CHECK(cudaMemset(p, 0, 256));
    // bytes 8..15: the wait limit (ns) of every bounded spin in device code (see common.cuh)
    const uint64_t limit = kDefaultWaitLimitNsHost;
    MINT_CUDA_CHECK(cudaMemcpy(static_cast<char*>(p) + 8, &limit, sizeof(limit), cudaMemcpyHostToDevice));
    g_status[device] = static_cast<uint32_t*>(p);
  }
  return g_status[device];
}

void set_wait_limit_ns(int device, uint64_t ns) {
  uint32_t* p = status_ptr(device);
  MINT_CHECK(ns > 0, "the wait limit must be positive");
  // synchronous copy: kernels launched after this call see the new limit
  MINT_CUDA_CHECK(cudaDeviceSynchronize());
  MINT_CUDA_CHECK(cudaMemcpy(reinterpret_cast<char*>(p) + 8, &ns, sizeof(ns), cudaMemcpyHostToDevice));
}

uint64_t wait_limit_ns(int device) {
  uint32_t* p = status_ptr(device);
  uint64_t ns = 0;
  MINT_CUDA_CHECK(cudaMemcpy(&ns, reinterpret_cast<char*>(p) + 8, sizeof(ns), cudaMemcpyDeviceToHost));
  return ns;
}

uint32_t read_status_word(int device, bool reset) {
  uint32_t* p = status_ptr(device);
  uint32_t v = 0;
  MINT_CUDA_CHECK(cudaMemcpy(&v, p, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  if (reset) MINT_CUDA_CHECK(cudaMemset(p, 0, sizeof(uint32_t)));
  return v;
}

int num_sms(int device) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sms[device] == 0) {
    int n = 0;
    MINT_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
    g_sms[device] = n;
  }
  return g_sms[device];
}

void check_smem_optin(int bytes, int device, const char* kernel) {
  int limit = 0;
  MINT_CUDA_CHECK(cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  MINT_CHECK(bytes <= limit, kernel, " needs ", bytes, " bytes of dynamic shared memory; the device allows ", limit);
}

CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                              uint32_t box_cols, bool swizzle128) {
  MINT_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  MINT_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes (ld=", ld, ")");
  CUtensorMap map;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  MINT_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", static_cast<int>(r), ") rows=", rows,
             " cols=", cols, " ld=", ld, " box=", box_rows, "x", box_cols);
  return map;
}

CUtensorMap make_tmap_2d(const void* base, int dtype, int esize, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint32_t box_rows, uint32_t box_cols, int swizzle) {
  MINT_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  MINT_CHECK((ld * esize) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * esize};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, static_cast<CUtensorMapDataType>(dtype), 2, const_cast<void*>(base), dims, strides,
                           box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, static_cast<CUtensorMapSwizzle>(swizzle),
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  MINT_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (store map) failed (", static_cast<int>(r), ")");
  return map;
}

CUtensorMap make_tmap_3d_bf16(const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                              uint64_t stride2, uint32_t box0, uint32_t box1, uint32_t box2, bool swizzle128) {
  MINT_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  MINT_CHECK((stride1 * 2) % 16 == 0 && (stride2 * 2) % 16 == 0, "TMA strides must be multiples of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1 * 2, stride2 * 2};
  cuuint32_t box[3] = {box0, box1, box2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  MINT_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3d) failed (", static_cast<int>(r), ")");
  return map;
}

CUtensorMap make_tmap_3d(const void* base, int dtype, int esize, uint64_t d0, uint64_t d1, uint64_t d2,
                         uint64_t stride1, uint64_t stride2, uint32_t box0, uint32_t box1, uint32_t box2, int swizzle) {
  MINT_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  MINT_CHECK((stride1 * esize) % 16 == 0 && (stride2 * esize) % 16 == 0, "TMA strides must be multiples of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1 * esize, stride2 * esize};
  cuuint32_t box[3] = {box0, box1, box2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&map, static_cast<CUtensorMapDataType>(dtype), 3, const_cast<void*>(base), dims, strides,
                           box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, static_cast<CUtensorMapSwizzle>(swizzle),
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  MINT_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3d) failed (", static_cast<int>(r), ") dims=", d0, "x", d1,
             "x", d2);
  return map;
}

CUtensorMap make_tmap_4d(const void* base, int dtype, int esize, const uint64_t (&dims)[4], const uint64_t (&strides)[3],
                         const uint32_t (&box)[4], int swizzle) {
  MINT_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  CUtensorMap map;
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t st[3];
  for (int i = 0; i < 3; ++i) {
    MINT_CHECK((strides[i] * esize) % 16 == 0, "TMA strides must be multiples of 16 bytes");
    st[i] = strides[i] * esize;
  }
  cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode_fn()(&map, static_cast<CUtensorMapDataType>(dtype), 4, const_cast<void*>(base), d, st, bx, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, static_cast<CUtensorMapSwizzle>(swizzle),
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  MINT_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (4d) failed (", static_cast<int>(r), ")");
  return map;
}

}  // namespace mint

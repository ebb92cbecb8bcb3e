// Allocation-free FlashAttention backward entry point (declared in flash_attn_bwd_noalloc.h; no
// counterpart in the reference framework). The fp32 dQ accumulator, the delta rows and a status
// block (status word + wait limit, the layout common.cuh defines) live in one file-scope device
// array instead of per-call allocations; the kernels are the ones of attention_bwd_sm100.cu,
// launched through flash_attn_bwd_launch_raw, and always report into that internal block. A small
// kernel then moves any error bits into the caller's status word when the caller passed one.
#include <cstdio>
#include <cstdint>
#include <exception>
#include <mutex>

#include "attention_bwd_raw.h"
#include "common.cuh"
#include "flash_attn_bwd_noalloc.h"

namespace {

constexpr long long kMaxRows = MINT_FLASH_ATTN_BWD_NOALLOC_MAX_ROWS;  // B * T * Hq
constexpr long long kHeadDim = 128;
constexpr long long kDqFloats = kMaxRows * kHeadDim;  // 16 MiB
constexpr long long kDeltaFloats = kMaxRows;          // 128 KiB
constexpr long long kStatusFloats = 64;               // 256 B status block: word 0 status, bytes 8..15 wait limit
constexpr long long kScratchFloats = kDqFloats + kDeltaFloats + kStatusFloats;
constexpr int kMaxDevices = 64;

}  // namespace

// One array per device, shared by every call on that device (see the header on overlapping calls).
static __device__ __align__(256) float g_fa_bwd_scratch[kScratchFloats];

namespace {

std::mutex g_setup_mu;
float* g_scratch_addr[kMaxDevices] = {};  // device address of g_fa_bwd_scratch, per device

void set_error(char* err, size_t len, const char* msg) {
  if (err != nullptr && len > 0) std::snprintf(err, len, "%s", msg);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Looks up the array's address on the current device (once per device). Host code must not pass
// `g_fa_bwd_scratch` itself to a kernel: on the host that name is only a stand-in symbol.
int scratch_for_current_device(float** out, char* err, size_t len) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error(err, len, "mint_flash_attn_bwd_noalloc: no usable current CUDA device");
    return 3;
  }
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_fa_bwd_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      char msg[256];
      std::snprintf(msg, sizeof(msg), "mint_flash_attn_bwd_noalloc: cudaGetSymbolAddress failed: %s",
                    cudaGetErrorString(e));
      set_error(err, len, msg);
      return 3;
    }
    mint::flash_attn_bwd_configure_current_device();  // throws on error (caught by the caller)
    // the status block's wait limit (a plain copy into the array; nothing is allocated)
    const uint64_t limit = mint::kDefaultWaitLimitNs;
    const size_t limit_off = static_cast<size_t>(kDqFloats + kDeltaFloats) * sizeof(float) + 8;
    e = cudaMemcpyToSymbol(g_fa_bwd_scratch, &limit, sizeof(limit), limit_off, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      char msg[256];
      std::snprintf(msg, sizeof(msg), "mint_flash_attn_bwd_noalloc: setting the wait limit failed: %s",
                    cudaGetErrorString(e));
      set_error(err, len, msg);
      return 3;
    }
    g_scratch_addr[dev] = static_cast<float*>(ptr);
  }
  *out = g_scratch_addr[dev];
  return 0;
}

// Moves the error bits of the internal status word into the caller's word and clears the former.
__global__ void forward_status_kernel(uint32_t* internal, uint32_t* user) {
  const uint32_t bits = *reinterpret_cast<volatile uint32_t*>(internal);
  if (bits != 0u) {
    atomicOr(user, bits);
    *internal = 0u;
  }
}

}  // namespace

extern "C" int mint_flash_attn_bwd_noalloc(const void* dout, const void* q, const void* k, const void* v,
                                           const void* o, const float* lse, const int* doc, void* dq, void* dk,
                                           void* dv, int B, int T, int Hq, int Hkv, int causal, int window,
                                           float scale, unsigned int* status, cudaStream_t stream, char* err,
                                           size_t err_len) {
  try {
    if (!dout || !q || !k || !v || !o || !lse || !dq || !dk || !dv) {
      set_error(err, err_len, "mint_flash_attn_bwd_noalloc: a required pointer is NULL");
      return 1;
    }
    if (B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0) {
      set_error(err, err_len, "mint_flash_attn_bwd_noalloc: need B, T, Hq, Hkv > 0 and Hq % Hkv == 0");
      return 1;
    }
    const void* bf16_bufs[8] = {dout, q, k, v, o, dq, dk, dv};
    for (const void* p : bf16_bufs) {
      if (!aligned16(p)) {
        set_error(err, err_len, "mint_flash_attn_bwd_noalloc: bf16 buffers must be 16-byte aligned");
        return 1;
      }
    }
    const long long rows = static_cast<long long>(B) * T * Hq;
    if (rows > kMaxRows) {
      char msg[256];
      std::snprintf(msg, sizeof(msg),
                    "mint_flash_attn_bwd_noalloc: B*T*Hq = %lld exceeds the static scratch limit of %lld rows",
                    rows, kMaxRows);
      set_error(err, err_len, msg);
      return 2;
    }
    float* base = nullptr;
    const int rc = scratch_for_current_device(&base, err, err_len);
    if (rc != 0) return rc;

    mint::FlashBwdRaw a{};
    a.dout = dout;
    a.q = q;
    a.k = k;
    a.v = v;
    a.o = o;
    a.lse = lse;
    a.doc = doc;
    a.dq = dq;
    a.dk = dk;
    a.dv = dv;
    a.dq_acc = base;
    a.delta = base + kDqFloats;
    // the kernels read their wait limit next to the status word, so they always get the internal
    // 256-byte block; a caller's 4-byte word receives the bits afterwards
    uint32_t* internal_status = reinterpret_cast<uint32_t*>(base + kDqFloats + kDeltaFloats);
    a.status = internal_status;
    a.B = B;
    a.T = T;
    a.Hq = Hq;
    a.Hkv = Hkv;
    a.causal = causal != 0;
    a.window = window;
    a.scale = scale;
    // the accumulator keeps the previous call's dQ: clear the rows this call uses
    cudaError_t e = cudaMemsetAsync(a.dq_acc, 0, static_cast<size_t>(rows * kHeadDim) * sizeof(float), stream);
    if (e != cudaSuccess) {
      char msg[256];
      std::snprintf(msg, sizeof(msg), "mint_flash_attn_bwd_noalloc: cudaMemsetAsync failed: %s",
                    cudaGetErrorString(e));
      set_error(err, err_len, msg);
      return 3;
    }
    mint::flash_attn_bwd_launch_raw(a, stream);
    if (status != nullptr) {
      forward_status_kernel<<<1, 1, 0, stream>>>(internal_status, reinterpret_cast<uint32_t*>(status));
      e = cudaGetLastError();
      if (e != cudaSuccess) {
        char msg[256];
        std::snprintf(msg, sizeof(msg), "mint_flash_attn_bwd_noalloc: status launch failed: %s",
                      cudaGetErrorString(e));
        set_error(err, err_len, msg);
        return 3;
      }
    }
    return 0;
  } catch (const std::exception& ex) {
    char msg[512];
    std::snprintf(msg, sizeof(msg), "mint_flash_attn_bwd_noalloc: %s", ex.what());
    set_error(err, err_len, msg);
    return 3;
  } catch (...) {
    set_error(err, err_len, "mint_flash_attn_bwd_noalloc: unknown error");
    return 3;
  }
}

extern "C" int mint_flash_attn_bwd_noalloc_status(int reset, unsigned int* out) {
  if (out == nullptr) return 1;
  float* base = nullptr;
  if (scratch_for_current_device(&base, nullptr, 0) != 0) return 3;
  const size_t off = static_cast<size_t>(kDqFloats + kDeltaFloats) * sizeof(float);
  // synchronous copies: the value reflects every call enqueued before this one has finished
  if (cudaDeviceSynchronize() != cudaSuccess) return 3;
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_fa_bwd_scratch, sizeof(v), off, cudaMemcpyDeviceToHost) != cudaSuccess) return 3;
  if (reset != 0 && v != 0) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_fa_bwd_scratch, &zero, sizeof(zero), off, cudaMemcpyHostToDevice) != cudaSuccess) {
      return 3;
    }
  }
  *out = v;
  return 0;
}

// Shared device helpers for the mint_b200 sm_100a kernels.
//
// * device status word: kernels never trap; on a timed-out wait or an invalid argument they
//   record an error code in a per-device status word (read by mint_b200.ops._ext.check_device_status)
//   and return.
// * bounded mbarrier waits (%globaltimer based), TMA (cp.async.bulk.tensor) loads, tcgen05
//   (UMMA) descriptors, MMA issue / commit and TMEM alloc / load, written as inline PTX.
#pragma once
#include <cmath>

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mint {

// ------------------------------------------------------------------------------------------
// status codes (bit flags OR-ed into the status word)
enum StatusCode : uint32_t {
  kStatusOk = 0,
  kStatusTimeoutProducer = 1u << 0,
  kStatusTimeoutMma = 1u << 1,
  kStatusTimeoutEpilogue = 1u << 2,
  kStatusBadArgument = 1u << 3,
  kStatusTimeoutPeer = 1u << 4,
  kStatusTimeoutAttention = 1u << 5,
};

// Per-device status block (256 bytes, allocated by host_common.cpp): word 0 is the status word
// (OR of StatusCode bits), bytes 8..15 the wait limit in nanoseconds that bounds every spin in
// device code. The host sets the limit at run time (mint_b200.ops._ext.set_wait_limit), so a test
// can make a wait give up after a fraction of a second; kDefaultWaitLimitNs applies when a kernel
// runs without a status block or the stored limit is zero.
constexpr uint64_t kDefaultWaitLimitNs = 4000000000ull;
constexpr int kStatusLimitWord = 2;  // uint32 index of the 64-bit limit inside the block

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint64_t wait_limit_ns(const uint32_t* status) {
  if (status == nullptr) return kDefaultWaitLimitNs;
  const uint64_t v = *reinterpret_cast<const volatile uint64_t*>(status + kStatusLimitWord);
  return v != 0 ? v : kDefaultWaitLimitNs;
}

// True when any kernel has recorded an error on this device: update kernels (AdamW, NorMuon) then
// leave the parameters untouched, so a step whose gradients came through a timed-out collective
// cannot corrupt the model before the host reads the word and raises.
__device__ __forceinline__ bool status_failed(const uint32_t* status) {
  return status != nullptr && *reinterpret_cast<const volatile uint32_t*>(status) != 0u;
}

// AdamW constants of one step: bias corrections folded into `step` = lr / (1 - b1^t) and
// `inv_bc2` = 1 / (1 - b2^t); `decay` = 1 - lr * wd (decoupled weight decay).
struct AdamWStep {
  float b1, b2, eps, step, decay, inv_bc2;
};

inline AdamWStep adamw_step_consts(double lr, double b1, double b2, double eps, double wd, long long t) {
  const double bc1 = 1.0 - std::pow(b1, static_cast<double>(t));
  const double bc2 = 1.0 - std::pow(b2, static_cast<double>(t));
  return AdamWStep{static_cast<float>(b1), static_cast<float>(b2), static_cast<float>(eps),
                   static_cast<float>(lr / bc1), static_cast<float>(1.0 - lr * wd), static_cast<float>(1.0 / bc2)};
}

// One element: m <- lerp(m, g, 1 - b1); v <- lerp(v, g^2, 1 - b2); returns the new parameter
// p * decay - step * m / (sqrt(v * inv_bc2) + eps).
__device__ __forceinline__ float adamw_elem(float p, float g, float& m, float& v, const AdamWStep& a) {
  m = m + (1.f - a.b1) * (g - m);
  v = v + (1.f - a.b2) * (g * g - v);
  return p * a.decay - a.step * m / (sqrtf(v * a.inv_bc2) + a.eps);
}

__device__ __forceinline__ void record_status(uint32_t* status, uint32_t code) {
  if (status != nullptr) atomicOr(status, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n.reg .b32 %%rx;\n.reg .pred %%px;\n"
      "elect.sync %%rx|%%px, %1;\n"
      "@%%px mov.s32 %0, 1;\n}"
      : "+r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}

// ------------------------------------------------------------------------------------------
// mbarrier
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
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` to complete. Returns false (and records `code`) when the
// wait exceeds the device's wait limit or `abort_flag` (shared) becomes non-zero.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status, uint32_t code,
                                          volatile int* abort_flag) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer();
  const uint64_t limit = wait_limit_ns(status);
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((it & 255u) == 0u) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (globaltimer() - t0 > limit) {
        record_status(status, code);
        if (abort_flag != nullptr) *abort_flag = 1;
        return false;
      }
    }
  }
}

// Whole-warp variant: every lane waits, and the result is made uniform across the warp (any lane
// failing fails all), so warp-collective tcgen05 instructions that follow never run diverged.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, uint32_t* status, uint32_t code,
                                               volatile int* abort_flag) {
  const bool ok = mbar_wait(bar, parity, status, code, abort_flag);
  return __all_sync(0xffffffffu, ok);
}

// ------------------------------------------------------------------------------------------
// TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// TMA store / reduce-add from shared memory (bulk-group completion)
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

__device__ __forceinline__ void tma_reduce_add_4d(const CUtensorMap* map, const void* src, int x, int y, int z, int w) {
  asm volatile("cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// at most N bulk groups of this thread still pending (their writes not yet performed)
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ------------------------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, accumulators in tensor memory)

// Shared-memory matrix descriptor for a 128B-swizzled canonical layout.
//   bits  0-13 start address >> 4, 16-29 leading byte offset >> 4, 32-45 stride byte offset >> 4,
//   bits 46-47 descriptor version (1 on sm_100), 49-51 base offset, 61-63 layout (2 = SWIZZLE_128B).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 x bf16 -> fp32, M x N tile.
//   bits 4-5 D format (1 = f32), 7-9 A format (1 = bf16), 10-12 B format (1 = bf16),
//   bit 15 A major (1 = MN-major), bit 16 B major, 17-22 N >> 3, 24-28 M >> 4.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// A operand read from tensor memory (P @ V in attention): [tmem_a] replaces the A descriptor.
__device__ __forceinline__ void umma_bf16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrive on `bar` when all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Whole-warp TMEM allocation; writes the base address to `*dst_smem`.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ------------------------------------------------------------------------------------------
// Thread-block clusters of 2 CTAs sharing one tcgen05 MMA (cta_group::2). No multicast anywhere:
// each CTA loads its own operand halves and every signal names its target CTA explicitly.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of `p` (an address in this CTA's shared memory) inside CTA `cta`.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t cta) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(cta));
  return out;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// mbarrier arrive on a barrier in another CTA of the cluster (address from mapa_shared).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// TMA load into this CTA's shared memory that completes its bytes on an mbarrier of either CTA
// of the pair (`bar_cluster` from mapa_shared).
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y,
                                                 int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// tcgen05.mma over a CTA pair: A rows split between the two CTAs' shared memory (same offsets),
// B columns split likewise, D = this pair's [256 x N] tile (128 rows in each CTA's tensor memory).
__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrive on the mbarrier at `bar_cluster` (either CTA of the pair) when this thread's pair MMAs complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}

// Paired TMEM allocation: one warp in each CTA (the same warp index) with the same slot offset.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ------------------------------------------------------------------------------------------
// Cross-GPU signalling over NVLink peer memory (symmetric buffers mapped into every rank).
// Flags carry a call sequence number and are never reset: a waiter waits for flag >= seq.
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
// generic-proxy global writes <-> async-proxy (TMA) global reads
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Spin (bounded by the device's wait limit) until *flag >= target. `sys` selects system scope (a
// flag written by another GPU) or GPU scope. Returns false and records `code` on timeout or abort.
__device__ __forceinline__ bool wait_flag(const int* flag, int target, bool sys, uint32_t* status, uint32_t code,
                                          volatile int* abort_flag) {
  if ((sys ? ld_acquire_sys(flag) : ld_acquire_gpu(flag)) >= target) return true;
  const uint64_t t0 = globaltimer();
  const uint64_t limit = wait_limit_ns(status);
  for (uint32_t it = 1;; ++it) {
    if ((sys ? ld_acquire_sys(flag) : ld_acquire_gpu(flag)) >= target) return true;
    if ((it & 63u) == 0u) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (globaltimer() - t0 > limit) {
        record_status(status, code);
        if (abort_flag != nullptr) *abort_flag = 1;
        return false;
      }
    }
  }
}

// 32 lanes x 32 columns of 32-bit: thread i of the warp receives row (lane base + i), 32 columns.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 16-byte vector reduction (fp32 add) into global memory.
__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// 32 lanes x 16 columns store into TMEM (thread i writes row lane base + i).
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 64 consecutive columns of one row per lane, as two 32-column stores
__device__ __forceinline__ void tmem_st_32x32b_x64(uint32_t taddr, const uint32_t (&r)[64]) {
  tmem_st_32x32b_x32(taddr, *reinterpret_cast<const uint32_t(*)[32]>(&r[0]));
  tmem_st_32x32b_x32(taddr + 32, *reinterpret_cast<const uint32_t(*)[32]>(&r[32]));
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------------------------------
// small math / conversion helpers
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

// 2^t for t <= 0 on the FMA pipe, for kernels whose exponentials would otherwise saturate the
// MUFU unit (attention softmax: one exponential per score). Cody-Waite range reduction: n = round(t)
// by adding 1.5 * 2^23 (the integer lands in the low mantissa bits), f = t - n in [-0.5, 0.5];
// 2^f from a degree-3 polynomial whose coefficients are a relative-error least-squares fit on 2000
// Chebyshev nodes of [-0.5, 0.5] (computed for this file with numpy; max relative error 7.8e-5,
// far below the bf16 rounding of the probabilities it feeds); 2^n added to the exponent bits.
// Returns 0 for t < -125 (and for -inf); a NaN argument comes back as NaN.
__device__ __forceinline__ float exp2_poly(float t) {
  const float tc = fmaxf(t, -125.f);
  const float j = tc + 12582912.f;  // 1.5 * 2^23: round to nearest integer
  const float n = j - 12582912.f;
  const float f = tc - n;
  float p = fmaf(0.05508868396282196f, f, 0.24260404706001282f);
  p = fmaf(p, f, 0.6932762265205383f);
  p = fmaf(p, f, 0.9999289512634277f);
  const int bits = __float_as_int(p) + ((__float_as_int(j) - 0x4B400000) << 23);
  // t >= -125 is false for NaN: such a t falls through to the last select and is returned as is
  return t >= -125.f ? __int_as_float(bits) : (t < -125.f ? 0.f : t);
}

// Packed fp32 pairs (Blackwell f32x2 instructions): one instruction for two lanes' worth of math.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rc, rd;\n"
      "mov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nmov.b64 rc, {%6, %7};\n"
      "fma.rn.f32x2 rd, ra, rb, rc;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\n"
      "mov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "add.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\n"
      "mov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "mul.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// 2^t for two arguments in one MUFU operation at bf16 precision: the arguments are rounded to bf16
// (one conversion instruction), the results come back packed as bf16x2 (lo in the low half), ready
// for a bf16 MMA operand. 2^-inf = +0. For softmax probabilities (t <= 0) the argument rounding
// costs at most ~0.2 % of p near p = 1/2 and less elsewhere -- the size of the bf16 rounding of p.
__device__ __forceinline__ uint32_t ex2_bf16x2(float lo, float hi) {
  uint32_t in, out;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(in) : "f"(hi), "f"(lo));
  asm("ex2.approx.ftz.bf16x2 %0, %1;" : "=r"(out) : "r"(in));
  return out;
}

// exact widening of a bf16x2 word to two floats
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

// Two finite floats to bf16x2 on the integer pipe: adding half a bf16 ulp (0x8000) to the
// sign-magnitude bit pattern and keeping the upper halves rounds the magnitude to nearest, ties
// away from zero (a carry into the exponent is the correct round-up); one PRMT packs both. Keeps the
// conversion off the pipe the exponentials use. Not for NaN / Inf inputs.
__device__ __forceinline__ uint32_t pack_bf16x2_int(float lo, float hi) {
  return __byte_perm(__float_as_uint(lo) + 0x8000u, __float_as_uint(hi) + 0x8000u, 0x7632);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}

}  // namespace mint

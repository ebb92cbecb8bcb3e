// ZeRO data-parallel collectives over NVLink peer memory (symmetric buffers mapped into every rank).
//
// zero_reduce_scatter: this rank's shard of sum over ranks of a flat fp32 gradient bucket, scaled by
//   1/dp, written into the shard buffer; the shard's squared norm is added to a device scalar (the
//   global gradient norm for clipping then needs one scalar all-reduce instead of a pass over the
//   shards). The kernel announces that its own bucket is final, waits for every peer's
//   announcement and pulls the peers' slices of its shard with 16-byte loads.
// zero_adamw_push: the sharded AdamW update with the all-gather fused in (new values stored to
//   every peer's copy as they are computed).
// zero_gather_pull: ZeRO-3's parameter gather, every rank's shard pulled into a local full buffer.
// zero_all_gather: pushes this rank's (updated) shard of a flat parameter bucket into every
//   peer's copy of the bucket; zero_barrier (one block, after the pushes of all buckets) announces
//   it and waits until every peer's shards have landed in this rank's copies.
// Flags hold a call sequence number and are never reset; every wait is bounded (common.cuh) and
// records kStatusTimeoutPeer in the device status word when it gives up.
// Reference: the per-parameter NCCL reduce_scatter_tensor / all_gather_into_tensor of
// mint/utils/parallel.py:237-261 and mint/optim/dist/muon_adamw.py:215-222.
#include <vector>

#include "common.cuh"
#include "host_common.h"

namespace mint {
namespace zc {

constexpr int kMaxRanks = 8;

struct Peers {
  const float* src[kMaxRanks];  // every rank's bucket (reduce-scatter) or shard destination (all-gather)
  float* dst[kMaxRanks];
  int* flag_peer[kMaxRanks];    // rank p's flag slot for this rank
};

// Announce (one thread of block 0) and wait (one thread per block) for every peer at `seq`.
__device__ __forceinline__ bool announce_and_wait(const Peers& pe, const int* flag_local, int rank, int world, int seq,
                                                  uint32_t* status, volatile int* abort_flag) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    __threadfence_system();
    for (int q = 0; q < world; ++q) {
      if (q != rank) st_release_sys(pe.flag_peer[q] + rank, seq);
    }
  }
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int q = 0; q < world && ok; ++q) {
      if (q != rank) ok = wait_flag(flag_local + q, seq, true, status, kStatusTimeoutPeer, abort_flag);
    }
    ok_s = ok ? 1 : 0;
  }
  __syncthreads();
  return ok_s != 0;
}

__global__ void __launch_bounds__(256) zero_reduce_scatter_kernel(Peers pe, float* __restrict__ shard, long long off,
                                                                  long long n, float scale, float* __restrict__ sumsq,
                                                                  const int* flag_local, int rank, int world, int seq,
                                                                  uint32_t* status) {
  __shared__ int abort_s;
  if (threadIdx.x == 0) abort_s = 0;
  __syncthreads();
  if (!announce_and_wait(pe, flag_local, rank, world, seq, status, &abort_s)) return;
  float acc = 0.f;
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < world; ++q) {
      const float4 v = reinterpret_cast<const float4*>(pe.src[q] + off)[i];
      t.x += v.x;
      t.y += v.y;
      t.z += v.z;
      t.w += v.w;
    }
    t.x *= scale;
    t.y *= scale;
    t.z *= scale;
    t.w *= scale;
    reinterpret_cast<float4*>(shard)[i] = t;
    acc += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
  }
  acc = warp_sum(acc);
  __shared__ float part[8];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0 && sumsq != nullptr) {
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += part[w];
    atomicAdd(sumsq, t);
  }
}

__global__ void __launch_bounds__(256) zero_push_kernel(Peers pe, const float* __restrict__ shard, long long off,
                                                        long long n, int rank, int world) {
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(shard)[i];
    for (int q = 0; q < world; ++q) {
      if (q != rank) reinterpret_cast<float4*>(pe.dst[q] + off)[i] = v;
    }
  }
}

// ZeRO-3 parameter gather: full[q * n .. (q + 1) * n) = rank q's shard (16-byte loads over NVLink
// from every peer's symmetric shard buffer, four in flight per thread). Shards change only in the
// optimizer step, which is fenced on both sides (see zero_gather_pull), so no flags are read here.
__global__ void __launch_bounds__(256) zero_gather_pull_kernel(Peers pe, float* __restrict__ full, long long n,
                                                               int world) {
  const long long n4 = n / 4;
  const long long total = n4 * world;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i0 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i0 < total; i0 += 4 * stride) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long i = i0 + u * stride;
      if (i < total) v[u] = reinterpret_cast<const float4*>(pe.src[i / n4])[i % n4];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long i = i0 + u * stride;
      if (i < total) reinterpret_cast<float4*>(full)[i] = v[u];
    }
  }
}

// Sharded AdamW fused with the parameter all-gather: each element of this rank's shard is updated
// once (p, m, v in local memory) and the new value is stored straight into every peer's copy of
// the bucket, so no separate push pass re-reads the shard. Gated on the status word like every
// update kernel: after a timed-out collective neither the local nor the peers' copies change.
__global__ void __launch_bounds__(256) zero_adamw_push_kernel(Peers pe, float* __restrict__ p,
                                                              const float* __restrict__ g, float* __restrict__ m,
                                                              float* __restrict__ v, long long off, long long n,
                                                              AdamWStep a, const float* __restrict__ gscale, int rank,
                                                              int world, const uint32_t* __restrict__ status) {
  if (status_failed(status)) return;
  const float gs = gscale != nullptr ? *gscale : 1.f;
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    const float4 gg = reinterpret_cast<const float4*>(g)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    pp.x = adamw_elem(pp.x, gg.x * gs, mm.x, vv.x, a);
    pp.y = adamw_elem(pp.y, gg.y * gs, mm.y, vv.y, a);
    pp.z = adamw_elem(pp.z, gg.z * gs, mm.z, vv.z, a);
    pp.w = adamw_elem(pp.w, gg.w * gs, mm.w, vv.w, a);
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    for (int q = 0; q < world; ++q) {
      if (q != rank) reinterpret_cast<float4*>(pe.dst[q] + off)[i] = pp;
    }
  }
}

// One block: the push kernel before it (stream order) has completed, so announce, then wait until
// every peer announced that its shard landed in this rank's bucket.
__global__ void zero_signal_kernel(Peers pe, const int* flag_local, int rank, int world, int seq, uint32_t* status) {
  __shared__ int abort_s;
  if (threadIdx.x == 0) abort_s = 0;
  __syncthreads();
  announce_and_wait(pe, flag_local, rank, world, seq, status, &abort_s);
}

}  // namespace zc

namespace {
zc::Peers make_peers(const std::vector<int64_t>& src, const std::vector<int64_t>& dst,
                     const std::vector<int64_t>& flags, int64_t world) {
  MINT_CHECK(world >= 2 && world <= zc::kMaxRanks, "fused ZeRO collectives need 2..8 ranks");
  zc::Peers pe{};
  for (int q = 0; q < world; ++q) {
    if (!src.empty()) pe.src[q] = reinterpret_cast<const float*>(src[q]);
    if (!dst.empty()) pe.dst[q] = reinterpret_cast<float*>(dst[q]);
    pe.flag_peer[q] = reinterpret_cast<int*>(flags[q]);
  }
  return pe;
}

int grid_for(long long n4, int dev) {
  const long long want = (n4 + 255) / 256;
  const long long cap = static_cast<long long>(num_sms(dev)) * 2;
  return static_cast<int>(std::max<long long>(1, std::min(want, cap)));
}
}  // namespace

// shard = scale * sum over ranks of bucket_p[rank * shard_len : (rank + 1) * shard_len]; sumsq += ||shard||^2.
void zero_reduce_scatter(const std::vector<int64_t>& bucket_ptrs, at::Tensor& shard, double scale,
                         const c10::optional<at::Tensor>& sumsq, const std::vector<int64_t>& flag_ptrs,
                         const at::Tensor& flags_local, int64_t rank, int64_t world, int64_t seq) {
  check_contig(shard, "shard");
  MINT_CHECK(shard.scalar_type() == at::kFloat && shard.numel() % 4 == 0, "shard must be fp32 with numel % 4 == 0");
  MINT_CHECK(static_cast<int64_t>(bucket_ptrs.size()) == world && static_cast<int64_t>(flag_ptrs.size()) == world,
             "one bucket / flag pointer per rank");
  c10::cuda::CUDAGuard guard(shard.device());
  const int dev = shard.get_device();
  zc::Peers pe = make_peers(bucket_ptrs, {}, flag_ptrs, world);
  const long long n = shard.numel();
  zc::zero_reduce_scatter_kernel<<<grid_for(n / 4, dev), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      pe, shard.data_ptr<float>(), rank * n, n, static_cast<float>(scale),
      sumsq.has_value() && sumsq->defined() ? sumsq->data_ptr<float>() : nullptr, flags_local.data_ptr<int>(),
      static_cast<int>(rank), static_cast<int>(world), static_cast<int>(seq), status_ptr(dev));
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

// Copy this rank's shard into every peer's bucket at offset rank * shard_len (bucket_ptrs[p] = rank p's
// bucket). Completion is published by zero_barrier, once after the pushes of every bucket.
void zero_all_gather(const at::Tensor& shard, const std::vector<int64_t>& bucket_ptrs, int64_t rank, int64_t world) {
  check_contig(shard, "shard");
  MINT_CHECK(shard.scalar_type() == at::kFloat && shard.numel() % 4 == 0, "shard must be fp32 with numel % 4 == 0");
  MINT_CHECK(static_cast<int64_t>(bucket_ptrs.size()) == world, "one bucket pointer per rank");
  c10::cuda::CUDAGuard guard(shard.device());
  const int dev = shard.get_device();
  std::vector<int64_t> no_flags(world, 0);
  zc::Peers pe = make_peers({}, bucket_ptrs, no_flags, world);
  const long long n = shard.numel();
  zc::zero_push_kernel<<<grid_for(n / 4, dev), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      pe, shard.data_ptr<float>(), rank * n, n, static_cast<int>(rank), static_cast<int>(world));
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

// ZeRO-3: full [world * n] fp32 = every rank's shard (shard_ptrs[q] = rank q's shard of n elements,
// in symmetric memory). The caller orders it after a zero_barrier that followed the last change of
// any shard, and no rank changes its shard before every peer's gathers have completed.
void zero_gather_pull(const std::vector<int64_t>& shard_ptrs, at::Tensor& full, int64_t rank, int64_t world) {
  check_contig(full, "full");
  MINT_CHECK(full.scalar_type() == at::kFloat && full.numel() % (4 * world) == 0,
             "full must be fp32 with numel a multiple of 4 x world");
  MINT_CHECK(static_cast<int64_t>(shard_ptrs.size()) == world, "one shard pointer per rank");
  for (int64_t q = 0; q < world; ++q) MINT_CHECK(shard_ptrs[q] % 16 == 0, "shards must be 16-byte aligned");
  (void)rank;
  c10::cuda::CUDAGuard guard(full.device());
  const int dev = full.get_device();
  std::vector<int64_t> no_flags(world, 0);
  zc::Peers pe = make_peers(shard_ptrs, {}, no_flags, world);
  const long long n = full.numel() / world;
  if (n == 0) return;
  zc::zero_gather_pull_kernel<<<grid_for(n * world / 16, dev), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      pe, full.data_ptr<float>(), n, static_cast<int>(world));
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

// AdamW on this rank's shard of a symmetric fp32 bucket (p = bucket_ptrs[rank] + rank * n) with the
// updated values pushed into every peer's bucket at the same offset; zero_barrier publishes them.
void zero_adamw_push(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v, double lr, double b1,
                     double b2, double eps, double wd, int64_t step, const c10::optional<at::Tensor>& gscale,
                     const std::vector<int64_t>& bucket_ptrs, int64_t rank, int64_t world) {
  const at::Tensor* all[4] = {&p, &g, &m, &v};
  for (const at::Tensor* t : all) {
    check_contig(*t, "adamw tensor");
    MINT_CHECK(t->scalar_type() == at::kFloat, "zero_adamw_push tensors must be fp32");
    MINT_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0, "zero_adamw_push tensors must be 16-byte aligned");
  }
  const long long n = p.numel();
  MINT_CHECK(n % 4 == 0 && g.numel() == n && m.numel() == n && v.numel() == n, "zero_adamw_push size mismatch");
  MINT_CHECK(static_cast<int64_t>(bucket_ptrs.size()) == world, "one bucket pointer per rank");
  MINT_CHECK(reinterpret_cast<int64_t>(p.data_ptr()) == bucket_ptrs[rank] + rank * n * 4,
             "p must be this rank's shard of its own symmetric bucket");
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(p.device());
  const int dev = p.get_device();
  std::vector<int64_t> no_flags(world, 0);
  zc::Peers pe = make_peers({}, bucket_ptrs, no_flags, world);
  zc::zero_adamw_push_kernel<<<grid_for(n / 4, dev), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      pe, p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), rank * n, n,
      adamw_step_consts(lr, b1, b2, eps, wd, step), gscale.has_value() ? gscale->data_ptr<float>() : nullptr,
      static_cast<int>(rank), static_cast<int>(world), status_ptr(dev));
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

// Stream-ordered barrier over the group: everything this rank's stream did before it (peer stores
// included) is visible to every peer when the peer's barrier returns.
void zero_barrier(const std::vector<int64_t>& flag_ptrs, const at::Tensor& flags_local, int64_t rank, int64_t world,
                  int64_t seq) {
  MINT_CHECK(static_cast<int64_t>(flag_ptrs.size()) == world, "one flag pointer per rank");
  c10::cuda::CUDAGuard guard(flags_local.device());
  const int dev = flags_local.get_device();
  zc::Peers pe = make_peers({}, {}, flag_ptrs, world);
  zc::zero_signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      pe, flags_local.data_ptr<int>(), static_cast<int>(rank), static_cast<int>(world), static_cast<int>(seq),
      status_ptr(dev));
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

}  // namespace mint

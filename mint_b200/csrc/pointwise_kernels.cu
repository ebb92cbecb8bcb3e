// Pointwise / gather / reduction kernels:
//   geglu            h = gelu_tanh(a) * b over the fused fc1||fc2 GEMM output, and its backward
//   embedding        (vocab-parallel) row gather and its scatter-add backward
//   cross-entropy    fused per-row log-sum-exp + in-place gradient logits (single GPU), or
//                    per-row statistics + in-place gradient for the vocab-parallel (TP) variant
//   adamw            fused decoupled-weight-decay Adam update over a flat fp32 shard
#include "common.cuh"
#include "host_common.h"

namespace mint {
namespace {

// gelu_tanh(x) = 0.5 x (1 + tanh(k0 (x + k1 x^3))),  k0 = sqrt(2/pi), k1 = 0.044715
constexpr float kGeluK0 = 0.7978845608028654f;
constexpr float kGeluK1 = 0.044715f;

__global__ void geglu_fwd_kernel(const __nv_bfloat16* __restrict__ ab, __nv_bfloat16* __restrict__ h, long long rows,
                                 int F) {
  const long long total = rows * F;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / F;
    const int c = static_cast<int>(i - r * F);
    const float a = __bfloat162float(ab[r * 2 * F + c]);
    const float b = __bfloat162float(ab[r * 2 * F + F + c]);
    const float t = tanhf(kGeluK0 * (a + kGeluK1 * a * a * a));
    h[i] = __float2bfloat16_rn(0.5f * a * (1.f + t) * b);
  }
}

__global__ void geglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ ab,
                                 __nv_bfloat16* __restrict__ dab, long long rows, int F) {
  const long long total = rows * F;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / F;
    const int c = static_cast<int>(i - r * F);
    const float a = __bfloat162float(ab[r * 2 * F + c]);
    const float b = __bfloat162float(ab[r * 2 * F + F + c]);
    const float g = __bfloat162float(dh[i]);
    const float u = kGeluK0 * (a + kGeluK1 * a * a * a);
    const float t = tanhf(u);
    const float gelu = 0.5f * a * (1.f + t);
    const float dgelu = 0.5f * (1.f + t) + 0.5f * a * (1.f - t * t) * kGeluK0 * (1.f + 3.f * kGeluK1 * a * a);
    dab[r * 2 * F + c] = __float2bfloat16_rn(g * b * dgelu);
    dab[r * 2 * F + F + c] = __float2bfloat16_rn(g * gelu);
  }
}

// 8 columns per thread with 16-byte loads / stores (F % 8 == 0)
__global__ void geglu_fwd_vec_kernel(const __nv_bfloat16* __restrict__ ab, __nv_bfloat16* __restrict__ h,
                                     long long rows, int F) {
  const int F8 = F >> 3;
  const long long total = rows * F8;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / F8;
    const int c = static_cast<int>(i - r * F8) << 3;
    const uint4 ua = *reinterpret_cast<const uint4*>(ab + r * 2 * F + c);
    const uint4 ub = *reinterpret_cast<const uint4*>(ab + r * 2 * F + F + c);
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&ua);
    const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&ub);
    uint4 out;
    uint32_t* po = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = __bfloat1622float2(pa[e]);
      const float2 b = __bfloat1622float2(pb[e]);
      const float t0 = tanhf(kGeluK0 * (a.x + kGeluK1 * a.x * a.x * a.x));
      const float t1 = tanhf(kGeluK0 * (a.y + kGeluK1 * a.y * a.y * a.y));
      po[e] = pack_bf16x2(0.5f * a.x * (1.f + t0) * b.x, 0.5f * a.y * (1.f + t1) * b.y);
    }
    *reinterpret_cast<uint4*>(h + r * F + c) = out;
  }
}

__global__ void geglu_bwd_vec_kernel(const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ ab,
                                     __nv_bfloat16* __restrict__ dab, long long rows, int F) {
  const int F8 = F >> 3;
  const long long total = rows * F8;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / F8;
    const int c = static_cast<int>(i - r * F8) << 3;
    const uint4 ua = *reinterpret_cast<const uint4*>(ab + r * 2 * F + c);
    const uint4 ub = *reinterpret_cast<const uint4*>(ab + r * 2 * F + F + c);
    const uint4 ug = *reinterpret_cast<const uint4*>(dh + r * F + c);
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&ua);
    const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&ub);
    const __nv_bfloat162* pg = reinterpret_cast<const __nv_bfloat162*>(&ug);
    uint4 oa, ob;
    uint32_t* qa = reinterpret_cast<uint32_t*>(&oa);
    uint32_t* qb = reinterpret_cast<uint32_t*>(&ob);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = __bfloat1622float2(pa[e]);
      const float2 b = __bfloat1622float2(pb[e]);
      const float2 g = __bfloat1622float2(pg[e]);
      float da[2], db[2];
      const float av[2] = {a.x, a.y}, bv[2] = {b.x, b.y}, gv[2] = {g.x, g.y};
#pragma unroll
      for (int z = 0; z < 2; ++z) {
        const float x = av[z];
        const float t = tanhf(kGeluK0 * (x + kGeluK1 * x * x * x));
        const float gelu = 0.5f * x * (1.f + t);
        const float dgelu = 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * kGeluK0 * (1.f + 3.f * kGeluK1 * x * x);
        da[z] = gv[z] * bv[z] * dgelu;
        db[z] = gv[z] * gelu;
      }
      qa[e] = pack_bf16x2(da[0], da[1]);
      qb[e] = pack_bf16x2(db[0], db[1]);
    }
    *reinterpret_cast<uint4*>(dab + r * 2 * F + c) = oa;
    *reinterpret_cast<uint4*>(dab + r * 2 * F + F + c) = ob;
  }
}

// one warp per token: out[m, :] = W[id - start, :] if the id is in this shard, else 0
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const float* __restrict__ w,
                                     float* __restrict__ out, int M, int D, long long start, long long rows) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  const long long local = ids[warp] - start;
  float* o = out + static_cast<long long>(warp) * D;
  if (local < 0 || local >= rows) {
    for (int j = lane; j < D; j += 32) o[j] = 0.f;
    return;
  }
  const float* src = w + local * D;
  if ((D & 3) == 0) {
    for (int j = lane * 4; j < D; j += 128) *reinterpret_cast<float4*>(o + j) = *reinterpret_cast<const float4*>(src + j);
  } else {
    for (int j = lane; j < D; j += 32) o[j] = src[j];
  }
}

template <typename T>
__global__ void embedding_bwd_kernel(const T* __restrict__ dout, const int64_t* __restrict__ ids,
                                     float* __restrict__ dw, int M, int D, long long start, long long rows) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  const long long local = ids[warp] - start;
  if (local < 0 || local >= rows) return;
  const T* g = dout + static_cast<long long>(warp) * D;
  float* dst = dw + local * D;
  for (int j = lane; j < D; j += 32) atomicAdd(dst + j, to_f32(g[j]));
}

// Block-wide reduction helpers (blockDim.x == 512).
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float x = lane < (blockDim.x >> 5) ? red[lane] : -INFINITY;
    x = warp_max(x);
    if (lane == 0) red[32] = x;
  }
  __syncthreads();
  const float r = red[32];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float x = lane < (blockDim.x >> 5) ? red[lane] : 0.f;
    x = warp_sum(x);
    if (lane == 0) red[32] = x;
  }
  __syncthreads();
  const float r = red[32];
  __syncthreads();
  return r;
}

constexpr float kLog2e = 1.4426950408889634f;

// Per-row max and sum-exp over the first `valid` columns of a bf16 row (8 elements per vector load).
__device__ __forceinline__ void max_sumexp8(const uint4& u, int j, int valid, float& mx, float& se) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
  float x[8];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(p[e]);
    x[2 * e] = f.x;
    x[2 * e + 1] = f.y;
  }
  float lm = -INFINITY;
#pragma unroll
  for (int e = 0; e < 8; ++e)
    if (j + e < valid) lm = fmaxf(lm, x[e]);
  if (lm > mx) {
    se *= exp2f((mx - lm) * kLog2e);
    mx = lm;
  }
#pragma unroll
  for (int e = 0; e < 8; ++e)
    if (j + e < valid) se += exp2f((x[e] - mx) * kLog2e);
}

// Row max and sum of exp(x - max) over the first `valid` columns. The vector path issues four
// 16-byte loads per thread before using any (64 KB in flight per 512-thread block), which keeps
// HBM streaming where one load at a time left it latency-bound.
__device__ __forceinline__ void row_max_sumexp(const __nv_bfloat16* __restrict__ row, int V, int valid, float* red,
                                               float& mx_out, float& se_out) {
  float mx = -INFINITY, se = 0.f;
  const bool vec = (V & 7) == 0;
  if (vec) {
    const int step = blockDim.x * 8;
    int j = threadIdx.x * 8;
    for (; j + 3 * step < V; j += 4 * step) {
      uint4 u[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) u[k] = *reinterpret_cast<const uint4*>(row + j + k * step);
#pragma unroll
      for (int k = 0; k < 4; ++k) max_sumexp8(u[k], j + k * step, valid, mx, se);
    }
    for (; j < V; j += step) max_sumexp8(*reinterpret_cast<const uint4*>(row + j), j, valid, mx, se);
  } else {
    for (int j = threadIdx.x; j < valid; j += blockDim.x) {
      const float x = __bfloat162float(row[j]);
      if (x > mx) {
        se *= exp2f((mx - x) * kLog2e);
        mx = x;
      }
      se += exp2f((x - mx) * kLog2e);
    }
  }
  const float gmx = block_max(mx, red);
  se = (mx == -INFINITY) ? 0.f : se * exp2f((mx - gmx) * kLog2e);
  se_out = block_sum(se, red);
  mx_out = gmx;
}

// grad[j] = (softmax_j - [j == t]) * scale for j < valid, 0 for padded columns; written in place.
__device__ __forceinline__ uint4 grad8(uint4 u, int j, int valid, float lse, long long t_local, float scale) {
  __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(p[e]);
    const int c0 = j + 2 * e, c1 = c0 + 1;
    float g0 = c0 < valid ? exp2f((f.x - lse) * kLog2e) : 0.f;
    float g1 = c1 < valid ? exp2f((f.y - lse) * kLog2e) : 0.f;
    if (c0 == t_local) g0 -= 1.f;
    if (c1 == t_local) g1 -= 1.f;
    p[e] = __floats2bfloat162_rn(g0 * scale, g1 * scale);
  }
  return u;
}

// softmax(x) - onehot(target), times `scale`, written over the row (four loads in flight per thread)
__device__ __forceinline__ void row_write_grad(__nv_bfloat16* __restrict__ row, int V, int valid, float lse,
                                               long long t_local, float scale) {
  const bool vec = (V & 7) == 0;
  if (vec) {
    const int step = blockDim.x * 8;
    int j = threadIdx.x * 8;
    for (; j + 3 * step < V; j += 4 * step) {
      uint4 u[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) u[k] = *reinterpret_cast<const uint4*>(row + j + k * step);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        *reinterpret_cast<uint4*>(row + j + k * step) = grad8(u[k], j + k * step, valid, lse, t_local, scale);
    }
    for (; j < V; j += step) {
      *reinterpret_cast<uint4*>(row + j) =
          grad8(*reinterpret_cast<const uint4*>(row + j), j, valid, lse, t_local, scale);
    }
  } else {
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
      float g = j < valid ? exp2f((__bfloat162float(row[j]) - lse) * kLog2e) : 0.f;
      if (j == t_local) g -= 1.f;
      row[j] = __float2bfloat16_rn(g * scale);
    }
  }
}

// Single-GPU fused CE: per row loss = lse - logit[target]; gradient logits written in place,
// scaled by mask[row] / denom. The second pass re-reads the row, which is still in L2.
__global__ void __launch_bounds__(512, 3) ce_fused_kernel(__nv_bfloat16* __restrict__ logits,
                                                       const int64_t* __restrict__ targets,
                                                       const float* __restrict__ mask, const float* __restrict__ denom,
                                                       float* __restrict__ row_loss, int M, int V, int valid,
                                                       long long vstart) {
  __shared__ float red[33];
  const int r = blockIdx.x;
  if (r >= M) return;
  __nv_bfloat16* row = logits + static_cast<long long>(r) * V;
  float mx, se;
  row_max_sumexp(row, V, valid, red, mx, se);
  const float lse = mx + logf(se);
  const long long t_local = targets[r] - vstart;
  float tl = 0.f;
  if (t_local >= 0 && t_local < valid) tl = __bfloat162float(row[t_local]);
  __syncthreads();
  if (threadIdx.x == 0) row_loss[r] = lse - tl;
  const float scale = mask[r] / *denom;
  row_write_grad(row, V, valid, lse, t_local, scale);
}

// TP pass 1: local max, local sum-exp relative to it, and the target logit if this shard owns it
__global__ void __launch_bounds__(512, 3) ce_stats_kernel(const __nv_bfloat16* __restrict__ logits,
                                                       const int64_t* __restrict__ targets, float* __restrict__ out_mx,
                                                       float* __restrict__ out_se, float* __restrict__ out_tl, int M,
                                                       int V, int valid, long long vstart) {
  __shared__ float red[33];
  const int r = blockIdx.x;
  if (r >= M) return;
  const __nv_bfloat16* row = logits + static_cast<long long>(r) * V;
  float mx, se;
  row_max_sumexp(row, V, valid, red, mx, se);
  if (threadIdx.x == 0) {
    const long long t_local = targets[r] - vstart;
    out_mx[r] = mx;
    out_se[r] = se;
    out_tl[r] = (t_local >= 0 && t_local < valid) ? __bfloat162float(row[t_local]) : 0.f;
  }
}

// TP pass 2: gradient logits in place given the global lse
__global__ void __launch_bounds__(512, 3) ce_grad_kernel(__nv_bfloat16* __restrict__ logits,
                                                      const int64_t* __restrict__ targets,
                                                      const float* __restrict__ mask, const float* __restrict__ lse,
                                                      const float* __restrict__ denom, int M, int V, int valid,
                                                      long long vstart) {
  const int r = blockIdx.x;
  if (r >= M) return;
  row_write_grad(logits + static_cast<long long>(r) * V, V, valid, lse[r], targets[r] - vstart, mask[r] / *denom);
}

// AdamW over a flat fp32 shard (adamw_elem, common.cuh).
// Skipped entirely (parameters and moments unchanged) once any kernel recorded an error status.
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, long long n, AdamWStep a, const float* __restrict__ gscale,
                             const uint32_t* __restrict__ status) {
  if (status_failed(status)) return;
  // gradient-clipping coefficient computed on the device (1 when the caller passes none)
  const float gs = gscale != nullptr ? *gscale : 1.f;
  const long long n4 = n / 4;
  float4* p4 = reinterpret_cast<float4*>(p);
  const float4* g4 = reinterpret_cast<const float4*>(g);
  float4* m4 = reinterpret_cast<float4*>(m);
  float4* v4 = reinterpret_cast<float4*>(v);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 pp = p4[i], gg = g4[i], mm = m4[i], vv = v4[i];
    pp.x = adamw_elem(pp.x, gg.x * gs, mm.x, vv.x, a);
    pp.y = adamw_elem(pp.y, gg.y * gs, mm.y, vv.y, a);
    pp.z = adamw_elem(pp.z, gg.z * gs, mm.z, vv.z, a);
    pp.w = adamw_elem(pp.w, gg.w * gs, mm.w, vv.w, a);
    p4[i] = pp;
    m4[i] = mm;
    v4[i] = vv;
  }
  for (long long i = n4 * 4 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float mi = m[i], vi = v[i];
    p[i] = adamw_elem(p[i], g[i] * gs, mi, vi, a);
    m[i] = mi;
    v[i] = vi;
  }
}

// Elementwise exp2_poly (common.cuh), exposed so its error bound and NaN handling can be tested
// against exp2f directly rather than only through attention's tolerances.
__global__ void exp2_poly_kernel(const float* __restrict__ x, float* __restrict__ y, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    y[i] = exp2_poly(x[i]);
}

int ew_grid(long long n, int dev) {
  const long long want = (n + 255) / 256;
  const long long cap = static_cast<long long>(num_sms(dev)) * 16;
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

}  // namespace

at::Tensor geglu_fwd(const at::Tensor& ab) {
  check_contig(ab, "ab");
  MINT_CHECK(ab.scalar_type() == at::kBFloat16, "geglu expects bf16");
  const int F = static_cast<int>(ab.size(-1) / 2);
  const long long rows = ab.numel() / (2 * F);
  auto sizes = ab.sizes().vec();
  sizes.back() = F;
  auto h = at::empty(sizes, ab.options());
  if (rows == 0) return h;
  c10::cuda::CUDAGuard g(ab.device());
  if (F % 8 == 0) {
    geglu_fwd_vec_kernel<<<ew_grid(rows * F / 8, ab.get_device()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(ab.data_ptr()), reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), rows, F);
  } else {
    geglu_fwd_kernel<<<ew_grid(rows * F, ab.get_device()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(ab.data_ptr()), reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), rows, F);
  }
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return h;
}

at::Tensor geglu_bwd(const at::Tensor& dh, const at::Tensor& ab) {
  check_contig(dh, "dh");
  check_contig(ab, "ab");
  MINT_CHECK(dh.scalar_type() == at::kBFloat16, "geglu grad must be bf16");
  const int F = static_cast<int>(ab.size(-1) / 2);
  const long long rows = ab.numel() / (2 * F);
  auto dab = at::empty_like(ab);
  if (rows == 0) return dab;
  c10::cuda::CUDAGuard g(ab.device());
  if (F % 8 == 0) {
    geglu_bwd_vec_kernel<<<ew_grid(rows * F / 8, ab.get_device()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dh.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(ab.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(dab.data_ptr()), rows, F);
  } else {
    geglu_bwd_kernel<<<ew_grid(rows * F, ab.get_device()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dh.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(ab.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(dab.data_ptr()), rows, F);
  }
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return dab;
}

at::Tensor embedding_fwd(const at::Tensor& ids, const at::Tensor& w, int64_t start) {
  check_contig(ids, "ids");
  check_contig(w, "weight");
  MINT_CHECK(ids.scalar_type() == at::kLong && w.scalar_type() == at::kFloat, "embedding: int64 ids, fp32 table");
  const int M = static_cast<int>(ids.numel());
  const int D = static_cast<int>(w.size(1));
  auto out = at::empty({M, D}, w.options());
  if (M == 0) return out;
  c10::cuda::CUDAGuard g(w.device());
  embedding_fwd_kernel<<<(M * 32 + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), w.data_ptr<float>(), out.data_ptr<float>(), M, D, start, w.size(0));
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return out;
}

at::Tensor embedding_bwd(const at::Tensor& dout, const at::Tensor& ids, int64_t rows, int64_t start) {
  check_contig(dout, "dout");
  check_contig(ids, "ids");
  const int M = static_cast<int>(ids.numel());
  const int D = static_cast<int>(dout.size(-1));
  auto dw = at::zeros({rows, D}, dout.options().dtype(at::kFloat));
  if (M == 0) return dw;
  c10::cuda::CUDAGuard g(dout.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = (M * 32 + 255) / 256;
  if (dout.scalar_type() == at::kFloat) {
    embedding_bwd_kernel<float><<<grid, 256, 0, st>>>(dout.data_ptr<float>(), ids.data_ptr<int64_t>(),
                                                      dw.data_ptr<float>(), M, D, start, rows);
  } else {
    MINT_CHECK(dout.scalar_type() == at::kBFloat16, "embedding grad must be fp32 or bf16");
    embedding_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), ids.data_ptr<int64_t>(), dw.data_ptr<float>(), M, D,
        start, rows);
  }
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return dw;
}

at::Tensor ce_fused_fwd_bwd(at::Tensor& logits, const at::Tensor& targets, const at::Tensor& mask,
                            const at::Tensor& denom, int64_t valid, int64_t vstart) {
  check_contig(logits, "logits");
  MINT_CHECK(logits.scalar_type() == at::kBFloat16 && logits.dim() == 2, "CE logits must be 2-D bf16");
  const int M = static_cast<int>(logits.size(0)), V = static_cast<int>(logits.size(1));
  MINT_CHECK(targets.numel() == M && mask.numel() == M, "CE targets/mask size mismatch");
  MINT_CHECK(valid >= 1 && valid <= V, "CE valid columns out of range");
  auto loss = at::empty({M}, logits.options().dtype(at::kFloat));
  if (M == 0) return loss;
  c10::cuda::CUDAGuard g(logits.device());
  ce_fused_kernel<<<M, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), targets.data_ptr<int64_t>(), mask.data_ptr<float>(),
      denom.data_ptr<float>(), loss.data_ptr<float>(), M, V, static_cast<int>(valid), vstart);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return loss;
}

std::vector<at::Tensor> ce_row_stats(const at::Tensor& logits, const at::Tensor& targets, int64_t valid,
                                     int64_t vstart) {
  check_contig(logits, "logits");
  const int M = static_cast<int>(logits.size(0)), V = static_cast<int>(logits.size(1));
  auto o = logits.options().dtype(at::kFloat);
  auto mx = at::empty({M}, o), se = at::empty({M}, o), tl = at::empty({M}, o);
  if (M == 0) return {mx, se, tl};
  c10::cuda::CUDAGuard g(logits.device());
  ce_stats_kernel<<<M, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), targets.data_ptr<int64_t>(), mx.data_ptr<float>(),
      se.data_ptr<float>(), tl.data_ptr<float>(), M, V, static_cast<int>(valid), vstart);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return {mx, se, tl};
}

void ce_grad_inplace(at::Tensor& logits, const at::Tensor& targets, const at::Tensor& mask, const at::Tensor& lse,
                     const at::Tensor& denom, int64_t valid, int64_t vstart) {
  check_contig(logits, "logits");
  const int M = static_cast<int>(logits.size(0)), V = static_cast<int>(logits.size(1));
  if (M == 0) return;
  c10::cuda::CUDAGuard g(logits.device());
  ce_grad_kernel<<<M, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), targets.data_ptr<int64_t>(), mask.data_ptr<float>(),
      lse.data_ptr<float>(), denom.data_ptr<float>(), M, V, static_cast<int>(valid), vstart);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void adamw_step(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v, double lr, double b1, double b2,
                double eps, double wd, int64_t step, const c10::optional<at::Tensor>& gscale) {
  const at::Tensor* all[4] = {&p, &g, &m, &v};
  for (const at::Tensor* t : all) {
    check_cuda(*t, "adamw tensor");
    MINT_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous(), "adamw tensors must be contiguous fp32");
    MINT_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0, "adamw tensors must be 16-byte aligned");
  }
  const long long n = p.numel();
  MINT_CHECK(g.numel() == n && m.numel() == n && v.numel() == n, "adamw size mismatch");
  if (n == 0) return;
  c10::cuda::CUDAGuard gd(p.device());
  adamw_kernel<<<ew_grid((n + 3) / 4, p.get_device()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), n,
      adamw_step_consts(lr, b1, b2, eps, wd, step), gscale.has_value() ? gscale->data_ptr<float>() : nullptr,
      status_ptr(p.get_device()));
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

at::Tensor exp2_poly_eval(const at::Tensor& x) {
  check_contig(x, "x");
  MINT_CHECK(x.scalar_type() == at::kFloat, "x must be fp32");
  auto y = at::empty_like(x);
  const long long n = x.numel();
  if (n == 0) return y;
  c10::cuda::CUDAGuard g(x.device());
  exp2_poly_kernel<<<ew_grid(n, x.get_device()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), y.data_ptr<float>(), n);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return y;
}

}  // namespace mint

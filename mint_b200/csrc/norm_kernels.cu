// Row-wise normalization kernels (memory bound, one warp per row, fp32 math):
//   rmsnorm           y = x * rsqrt(mean(x^2) + eps) * (1 + scale)
//   add_rmsnorm       h = res + bf16(rmsnorm(a; post)),  y = rmsnorm(h; pre)   (sandwich-norm block update)
//   qk_norm_rope      per-head RMSNorm of q and k + half-split rotary embedding, splitting the fused QKV output
// Backward kernels reduce the scale gradients per CTA in shared memory, then one atomicAdd per
// column per CTA into an fp32 accumulator.
#include <cstdlib>
#include <type_traits>

#include "common.cuh"
#include "host_common.h"

namespace mint {
namespace {

constexpr int kRowsPerBlock = 8;  // 8 warps
constexpr int kMaxD = 4096;

template <typename Tin, typename Tout>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const Tin* __restrict__ x, const float* __restrict__ scale,
                                                          Tout* __restrict__ y, float* __restrict__ rstd_out, int rows,
                                                          int D, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowsPerBlock + warp;
  if (row >= rows) return;
  const Tin* xr = x + static_cast<long long>(row) * D;
  float ss = 0.f;
  for (int j = lane; j < D; j += 32) {
    const float v = to_f32(xr[j]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / D + eps);
  Tout* yr = y + static_cast<long long>(row) * D;
  for (int j = lane; j < D; j += 32) yr[j] = from_f32<Tout>(to_f32(xr[j]) * r * (1.f + scale[j]));
  if (lane == 0) rstd_out[row] = r;
}

// dx = r * w * dy - x * r^3 * mean(dy * w * x);  dscale += dy * x * r
template <typename Tin, typename Tdy, typename Tdx>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const Tdy* __restrict__ dy, const Tin* __restrict__ x,
                                                          const float* __restrict__ rstd,
                                                          const float* __restrict__ scale, Tdx* __restrict__ dx,
                                                          float* __restrict__ dscale, int rows, int D) {
  extern __shared__ float s_ds[];  // [nwarps][D], each lane owns distinct columns of its warp's row
  const int nwarps = blockDim.x >> 5;
  for (int j = threadIdx.x; j < nwarps * D; j += blockDim.x) s_ds[j] = 0.f;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* my = s_ds + warp * D;
  for (int row = blockIdx.x * nwarps + warp; row < rows; row += gridDim.x * nwarps) {
    const Tin* xr = x + static_cast<long long>(row) * D;
    const Tdy* dyr = dy + static_cast<long long>(row) * D;
    const float r = rstd[row];
    float dot = 0.f;
    for (int j = lane; j < D; j += 32) dot += to_f32(dyr[j]) * (1.f + scale[j]) * to_f32(xr[j]);
    dot = warp_sum(dot) / D;
    Tdx* dxr = dx + static_cast<long long>(row) * D;
    for (int j = lane; j < D; j += 32) {
      const float xv = to_f32(xr[j]), g = to_f32(dyr[j]);
      dxr[j] = from_f32<Tdx>(r * (1.f + scale[j]) * g - xv * r * r * r * dot);
      my[j] += g * xv * r;
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    float t = 0.f;
    for (int w = 0; w < nwarps; ++w) t += s_ds[w * D + j];
    atomicAdd(&dscale[j], t);
  }
}

// h = res + bf16(rms(a) * (1 + post));  y = rms(h) * (1 + pre)  (y optional)
template <typename Ty>
__global__ void __launch_bounds__(256) add_rmsnorm_fwd_kernel(const float* __restrict__ res,
                                                              const __nv_bfloat16* __restrict__ a,
                                                              const float* __restrict__ post,
                                                              const float* __restrict__ pre, float* __restrict__ h,
                                                              Ty* __restrict__ y, float* __restrict__ rstd_a,
                                                              float* __restrict__ rstd_h, int rows, int D, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowsPerBlock + warp;
  if (row >= rows) return;
  const long long off = static_cast<long long>(row) * D;
  float ss = 0.f;
  for (int j = lane; j < D; j += 32) {
    const float v = __bfloat162float(a[off + j]);
    ss += v * v;
  }
  const float ra = rsqrtf(warp_sum(ss) / D + eps);
  float sh = 0.f;
  for (int j = lane; j < D; j += 32) {
    const float n = __bfloat162float(__float2bfloat16_rn(__bfloat162float(a[off + j]) * ra * (1.f + post[j])));
    const float hv = res[off + j] + n;
    h[off + j] = hv;
    sh += hv * hv;
  }
  if (lane == 0) rstd_a[row] = ra;
  if (pre != nullptr) {
    const float rh = rsqrtf(warp_sum(sh) / D + eps);
    __syncwarp();
    for (int j = lane; j < D; j += 32) y[off + j] = from_f32<Ty>(h[off + j] * rh * (1.f + pre[j]));
    if (lane == 0) rstd_h[row] = rh;
  }
}

__device__ __forceinline__ float half_warp_sum(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void unpack_bf16x8(const uint4& raw, float (&x)[8]) {
  const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(h2[e]);
    x[2 * e] = f.x;
    x[2 * e + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float (&x)[8]) {
  return make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]), pack_bf16x2(x[4], x[5]),
                    pack_bf16x2(x[6], x[7]));
}

__device__ __forceinline__ void load_f32x8(const float* p, float (&x)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
}

// Register-resident add + RMSNorm forward for D = 32 * VPT (VPT a multiple of 8): one warp per
// row, lane l owns columns {l * 8 + 256 * c + e}; the row's a (bf16) and res (fp32) are loaded with
// 16-byte accesses before any math (144 B in flight per lane at D = 768), h and y written once.
template <int VPT, typename Ty>
__global__ void __launch_bounds__(256) add_rmsnorm_fwd_reg_kernel(
    const float* __restrict__ res, const __nv_bfloat16* __restrict__ a, const float* __restrict__ post,
    const float* __restrict__ pre, float* __restrict__ h, Ty* __restrict__ y, float* __restrict__ rstd_a,
    float* __restrict__ rstd_h, int rows, float eps) {
  constexpr int D = VPT * 32;
  constexpr int NC = VPT / 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowsPerBlock + warp;
  if (row >= rows) return;
  const long long off = static_cast<long long>(row) * D;
  uint4 araw[NC];
  float4 r0[NC], r1[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int j = lane * 8 + c * 256;
    araw[c] = *reinterpret_cast<const uint4*>(a + off + j);
    r0[c] = *reinterpret_cast<const float4*>(res + off + j);
    r1[c] = *reinterpret_cast<const float4*>(res + off + j + 4);
  }
  float av[VPT];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&araw[c]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(b2[e]);
      av[c * 8 + 2 * e] = f.x;
      av[c * 8 + 2 * e + 1] = f.y;
      ss += f.x * f.x + f.y * f.y;
    }
  }
  const float ra = rsqrtf(warp_sum(ss) * (1.f / D) + eps);
  float sh = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int j = lane * 8 + c * 256;
    const float rv[8] = {r0[c].x, r0[c].y, r0[c].z, r0[c].w, r1[c].x, r1[c].y, r1[c].z, r1[c].w};
    float pw[8];
    load_f32x8(post + j, pw);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      // the normalized branch is rounded to bf16 as the unfused module's output would be
      const float n = __bfloat162float(__float2bfloat16_rn(av[c * 8 + e] * ra * (1.f + pw[e])));
      av[c * 8 + e] = rv[e] + n;  // av now holds h
      sh += av[c * 8 + e] * av[c * 8 + e];
    }
    *reinterpret_cast<float4*>(h + off + j) = make_float4(av[c * 8], av[c * 8 + 1], av[c * 8 + 2], av[c * 8 + 3]);
    *reinterpret_cast<float4*>(h + off + j + 4) =
        make_float4(av[c * 8 + 4], av[c * 8 + 5], av[c * 8 + 6], av[c * 8 + 7]);
  }
  if (lane == 0) rstd_a[row] = ra;
  if (pre == nullptr) return;
  const float rh = rsqrtf(warp_sum(sh) * (1.f / D) + eps);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int j = lane * 8 + c * 256;
    float pw[8], o[8];
    load_f32x8(pre + j, pw);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = av[c * 8 + e] * rh * (1.f + pw[e]);
    if constexpr (std::is_same<Ty, float>::value) {
      *reinterpret_cast<float4*>(y + off + j) = make_float4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<float4*>(y + off + j + 4) = make_float4(o[4], o[5], o[6], o[7]);
    } else {
      *reinterpret_cast<uint4*>(y + off + j) = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]),
                                                          pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
    }
  }
  if (lane == 0) rstd_h[row] = rh;
}

// dres = dh + rmsnorm_bwd(dy; h, pre);  da = rmsnorm_bwd(dres; a, post)
template <typename Ty>
__global__ void __launch_bounds__(256) add_rmsnorm_bwd_kernel(
    const float* __restrict__ dh, const Ty* __restrict__ dy, const __nv_bfloat16* __restrict__ a,
    const float* __restrict__ h, const float* __restrict__ rstd_a, const float* __restrict__ rstd_h,
    const float* __restrict__ post, const float* __restrict__ pre, float* __restrict__ dres,
    __nv_bfloat16* __restrict__ da, float* __restrict__ dpost, float* __restrict__ dpre, int rows, int D) {
  extern __shared__ float s_acc[];  // [nwarps][2 * D]: dpost, dpre per warp
  const int nwarps = blockDim.x >> 5;
  for (int j = threadIdx.x; j < nwarps * 2 * D; j += blockDim.x) s_acc[j] = 0.f;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* my = s_acc + warp * 2 * D;
  for (int row = blockIdx.x * nwarps + warp; row < rows; row += gridDim.x * nwarps) {
    const long long off = static_cast<long long>(row) * D;
    // 1) gradient into h: dh + d(y)/d(h)
    if (dy != nullptr && pre != nullptr) {
      const float rh = rstd_h[row];
      float dot = 0.f;
      for (int j = lane; j < D; j += 32) dot += to_f32(dy[off + j]) * (1.f + pre[j]) * h[off + j];
      dot = warp_sum(dot) / D;
      for (int j = lane; j < D; j += 32) {
        const float g = to_f32(dy[off + j]), hv = h[off + j];
        const float v = rh * (1.f + pre[j]) * g - hv * rh * rh * rh * dot + (dh != nullptr ? dh[off + j] : 0.f);
        dres[off + j] = v;
        my[D + j] += g * hv * rh;
      }
    } else {
      for (int j = lane; j < D; j += 32) dres[off + j] = dh != nullptr ? dh[off + j] : 0.f;
    }
    __syncwarp();
    // 2) gradient into a through the post norm (dn = dres)
    const float ra = rstd_a[row];
    float dot = 0.f;
    for (int j = lane; j < D; j += 32) dot += dres[off + j] * (1.f + post[j]) * __bfloat162float(a[off + j]);
    dot = warp_sum(dot) / D;
    for (int j = lane; j < D; j += 32) {
      const float g = dres[off + j], av = __bfloat162float(a[off + j]);
      da[off + j] = __float2bfloat16_rn(ra * (1.f + post[j]) * g - av * ra * ra * ra * dot);
      my[j] += g * av * ra;
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    float tp = 0.f, tq = 0.f;
    for (int w = 0; w < nwarps; ++w) {
      tp += s_acc[w * 2 * D + j];
      tq += s_acc[w * 2 * D + D + j];
    }
    atomicAdd(&dpost[j], tp);
    if (dpre != nullptr) atomicAdd(&dpre[j], tq);
  }
}

// Register-resident add + RMSNorm backward for D = 32 * VPT (VPT a multiple of 8), 4 warps per
// block, one warp per row: every operand of the row (dy, h, dh, a and both rstd values) is loaded
// with 16-byte accesses before the first reduction, so ~290 B per lane are in flight at D = 768.
// The (1 + scale) weights and the per-warp scale-gradient accumulators live in shared memory, which
// keeps the kernel near 100 registers (5 blocks per SM).
constexpr int kArnBwdWarps = 4;
template <int VPT>
__global__ void __launch_bounds__(kArnBwdWarps * 32) add_rmsnorm_bwd_reg_kernel(
    const float* __restrict__ dh, const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ a,
    const float* __restrict__ h, const float* __restrict__ rstd_a, const float* __restrict__ rstd_h,
    const float* __restrict__ post, const float* __restrict__ pre, float* __restrict__ dres,
    __nv_bfloat16* __restrict__ da, float* __restrict__ dpost, float* __restrict__ dpre, int rows) {
  constexpr int D = VPT * 32;
  constexpr int NC = VPT / 8;
  // shared arrays are indexed [i][lane] (i = c * 8 + e, the lane's i-th column) so that a warp's
  // 32 accesses hit 32 different banks
  __shared__ float s_w[2][VPT][32];                  // 1 + post, 1 + pre
  __shared__ float s_acc[kArnBwdWarps][2][VPT][32];  // per-warp dpost, dpre column sums
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    const int i = (j >> 8) * 8 + (j & 7), l = (j & 255) >> 3;
    s_w[0][i][l] = 1.f + post[j];
    s_w[1][i][l] = pre != nullptr ? 1.f + pre[j] : 1.f;
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    s_acc[warp][0][i][lane] = 0.f;
    s_acc[warp][1][i][lane] = 0.f;
  }
  __syncthreads();
  for (int row = blockIdx.x * kArnBwdWarps + warp; row < rows; row += gridDim.x * kArnBwdWarps) {
    const long long off = static_cast<long long>(row) * D;
    uint4 yraw[NC], araw[NC];
    float4 h0[NC], h1[NC], d0[NC], d1[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int j = lane * 8 + c * 256;
      if (dy != nullptr) {
        yraw[c] = *reinterpret_cast<const uint4*>(dy + off + j);
        h0[c] = *reinterpret_cast<const float4*>(h + off + j);
        h1[c] = *reinterpret_cast<const float4*>(h + off + j + 4);
      }
      if (dh != nullptr) {
        d0[c] = *reinterpret_cast<const float4*>(dh + off + j);
        d1[c] = *reinterpret_cast<const float4*>(dh + off + j + 4);
      } else {
        d0[c] = d1[c] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      araw[c] = *reinterpret_cast<const uint4*>(a + off + j);
    }
    const float ra = rstd_a[row];
    const float rh = dy != nullptr ? rstd_h[row] : 0.f;
    float g[VPT];  // gradient into h = dres
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const float dv[8] = {d0[c].x, d0[c].y, d0[c].z, d0[c].w, d1[c].x, d1[c].y, d1[c].z, d1[c].w};
#pragma unroll
      for (int e = 0; e < 8; ++e) g[c * 8 + e] = dv[e];
    }
    if (dy != nullptr) {
      float yv[VPT], hv[VPT];
      float dot = 0.f;
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int j = lane * 8 + c * 256;
        const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&yraw[c]);
        const float hh[8] = {h0[c].x, h0[c].y, h0[c].z, h0[c].w, h1[c].x, h1[c].y, h1[c].z, h1[c].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(b2[e]);
          yv[c * 8 + 2 * e] = f.x;
          yv[c * 8 + 2 * e + 1] = f.y;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          hv[c * 8 + e] = hh[e];
          dot += yv[c * 8 + e] * s_w[1][c * 8 + e][lane] * hh[e];
        }
      }
      dot = warp_sum(dot) * (1.f / D);
      const float k3 = rh * rh * rh * dot;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        g[i] += rh * s_w[1][i][lane] * yv[i] - hv[i] * k3;
        s_acc[warp][1][i][lane] += yv[i] * hv[i] * rh;
      }
    }
    float av[VPT];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int j = lane * 8 + c * 256;
      *reinterpret_cast<float4*>(dres + off + j) = make_float4(g[c * 8], g[c * 8 + 1], g[c * 8 + 2], g[c * 8 + 3]);
      *reinterpret_cast<float4*>(dres + off + j + 4) =
          make_float4(g[c * 8 + 4], g[c * 8 + 5], g[c * 8 + 6], g[c * 8 + 7]);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&araw[c]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(b2[e]);
        av[c * 8 + 2 * e] = f.x;
        av[c * 8 + 2 * e + 1] = f.y;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) dot += g[c * 8 + e] * s_w[0][c * 8 + e][lane] * av[c * 8 + e];
    }
    dot = warp_sum(dot) * (1.f / D);
    const float k3 = ra * ra * ra * dot;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int j = lane * 8 + c * 256;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int i = c * 8 + e;
        o[e] = ra * s_w[0][i][lane] * g[i] - av[i] * k3;
        s_acc[warp][0][i][lane] += g[i] * av[i] * ra;
      }
      *reinterpret_cast<uint4*>(da + off + j) = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]),
                                                           pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    const int i = (j >> 8) * 8 + (j & 7), l = (j & 255) >> 3;
    float tp = 0.f, tq = 0.f;
#pragma unroll
    for (int w = 0; w < kArnBwdWarps; ++w) {
      tp += s_acc[w][0][i][l];
      tq += s_acc[w][1][i][l];
    }
    atomicAdd(&dpost[j], tp);
    if (dpre != nullptr) atomicAdd(&dpre[j], tq);
  }
}

// Register-resident rmsnorm_bwd for fp32 x, bf16 dy, fp32 dx and D = 32 * VPT <= 768 (VPT a
// multiple of 8): one warp per row, lane l owns columns {l * 8 + 256 * c + e}, 16-byte vector loads,
// each operand read once, the scale gradient accumulated in registers across rows.
template <int VPT>
__global__ void __launch_bounds__(256) rmsnorm_bwd_reg_kernel(const __nv_bfloat16* __restrict__ dy,
                                                              const float* __restrict__ x,
                                                              const float* __restrict__ rstd,
                                                              const float* __restrict__ scale, float* __restrict__ dx,
                                                              float* __restrict__ dscale, int rows) {
  constexpr int D = VPT * 32;
  constexpr int NC = VPT / 8;
  __shared__ float s_red[8][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float w1[VPT], acc[VPT];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      w1[c * 8 + e] = 1.f + scale[lane * 8 + c * 256 + e];
      acc[c * 8 + e] = 0.f;
    }
  }
  const int nwarps = blockDim.x >> 5;
  for (int row = blockIdx.x * nwarps + warp; row < rows; row += gridDim.x * nwarps) {
    const long long off = static_cast<long long>(row) * D;
    float g[VPT], xv[VPT];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int j = lane * 8 + c * 256;
      const uint4 u = *reinterpret_cast<const uint4*>(dy + off + j);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(b2[e]);
        g[c * 8 + 2 * e] = f.x;
        g[c * 8 + 2 * e + 1] = f.y;
      }
      const float4 x0 = *reinterpret_cast<const float4*>(x + off + j);
      const float4 x1 = *reinterpret_cast<const float4*>(x + off + j + 4);
      xv[c * 8 + 0] = x0.x; xv[c * 8 + 1] = x0.y; xv[c * 8 + 2] = x0.z; xv[c * 8 + 3] = x0.w;
      xv[c * 8 + 4] = x1.x; xv[c * 8 + 5] = x1.y; xv[c * 8 + 6] = x1.z; xv[c * 8 + 7] = x1.w;
    }
    const float r = rstd[row];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) dot += g[i] * w1[i] * xv[i];
    dot = warp_sum(dot) * (1.f / D);
    const float k3 = r * r * r * dot;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float d[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int i = c * 8 + e;
        d[e] = r * w1[i] * g[i] - xv[i] * k3;
        acc[i] += g[i] * xv[i] * r;
      }
      const int j = lane * 8 + c * 256;
      *reinterpret_cast<float4*>(dx + off + j) = make_float4(d[0], d[1], d[2], d[3]);
      *reinterpret_cast<float4*>(dx + off + j + 4) = make_float4(d[4], d[5], d[6], d[7]);
    }
  }
#pragma unroll
  for (int c = 0; c < NC; ++c) {
#pragma unroll
    for (int e = 0; e < 8; ++e) s_red[warp][lane * 8 + c * 256 + e] = acc[c * 8 + e];
  }
  __syncthreads();
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    float t = 0.f;
    for (int w = 0; w < nwarps; ++w) t += s_red[w][j];
    atomicAdd(&dscale[j], t);
  }
}

// One warp per (token, head) row of q or k; v heads are copied. Rows ordered token-major.
// qkv [M, (Hq + 2 Hkv) * Dh]; q [M, Hq, Dh]; k, v [M, Hkv, Dh]. Position of token m = start + (m % T).
__global__ void __launch_bounds__(256) qk_norm_rope_fwd_kernel(
    const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ qs, const float* __restrict__ ks,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, __nv_bfloat16* __restrict__ q,
    __nv_bfloat16* __restrict__ k, __nv_bfloat16* __restrict__ v, float* __restrict__ rq, float* __restrict__ rk,
    int M, int T, int Hq, int Hkv, int Dh, int start, int use_rope, float eps) {
  extern __shared__ float s_row[];  // [8][Dh]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = Hq + 2 * Hkv;
  const long long item = static_cast<long long>(blockIdx.x) * kRowsPerBlock + warp;
  if (item >= static_cast<long long>(M) * H) return;
  const int m = static_cast<int>(item / H);
  const int hh = static_cast<int>(item % H);
  const __nv_bfloat16* src = qkv + static_cast<long long>(m) * H * Dh + static_cast<long long>(hh) * Dh;
  if (hh >= Hq + Hkv) {  // v: copy
    __nv_bfloat16* dst = v + (static_cast<long long>(m) * Hkv + (hh - Hq - Hkv)) * Dh;
    for (int j = lane; j < Dh; j += 32) dst[j] = src[j];
    return;
  }
  const bool is_q = hh < Hq;
  const float* sc = is_q ? qs : ks;
  float* buf = s_row + warp * Dh;
  float ss = 0.f;
  for (int j = lane; j < Dh; j += 32) {
    const float x = __bfloat162float(src[j]);
    ss += x * x;
  }
  const float r = rsqrtf(warp_sum(ss) / Dh + eps);
  for (int j = lane; j < Dh; j += 32) buf[j] = __bfloat162float(src[j]) * r * (1.f + sc[j]);
  __syncwarp();
  __nv_bfloat16* dst = is_q ? q + (static_cast<long long>(m) * Hq + hh) * Dh
                            : k + (static_cast<long long>(m) * Hkv + (hh - Hq)) * Dh;
  const int half = Dh / 2;
  const int pos = start + (m % T);
  for (int j = lane; j < Dh; j += 32) {
    float out = buf[j];
    if (use_rope) {
      const int i = j < half ? j : j - half;
      const float c = cos_t[static_cast<long long>(pos) * half + i];
      const float s = sin_t[static_cast<long long>(pos) * half + i];
      out = j < half ? buf[j] * c - buf[j + half] * s : buf[j - half] * s + buf[j] * c;
    }
    dst[j] = __float2bfloat16_rn(out);
  }
  if (lane == 0) (is_q ? rq : rk)[static_cast<long long>(m) * (is_q ? Hq : Hkv) + (is_q ? hh : hh - Hq)] = r;
}

// head_dim 128 specializations. A half-warp owns one 256-byte row: lane l (0..15 within the
// half-warp) holds elements 8l..8l+7 (16-byte accesses) and its rotation partner (j +- 64) is lane
// l ^ 8 of the same half-warp; reductions stay inside the half-warp (xor 8, 4, 2, 1). Each thread
// issues the loads of all its rows before any math, so an SM keeps 64-128 KB of reads in flight,
// which is what HBM3e needs to stream at full rate (one 8-byte load per thread reached ~40 %).
constexpr int kQkFwdRows = 4;  // rows per half-warp, forward

// Block (x, hh) handles head slot hh (q, k or v) of rows m = x*16*R + i*16 + hw (i < R): each row
// is 256 contiguous bytes, so fixing the head per block costs no coalescing and needs no division.
__global__ void __launch_bounds__(256) qk_norm_rope_fwd128_kernel(
    const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ qs, const float* __restrict__ ks,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, __nv_bfloat16* __restrict__ q,
    __nv_bfloat16* __restrict__ k, __nv_bfloat16* __restrict__ v, float* __restrict__ rq, float* __restrict__ rk,
    int M, int T, int Hq, int Hkv, int start, int use_rope, float eps) {
  constexpr int Dh = 128;
  const int hw = threadIdx.x >> 4, hl = threadIdx.x & 15;
  const int hh = blockIdx.y;
  const int H = Hq + 2 * Hkv;
  const long long rstride = static_cast<long long>(H) * Dh;
  const int m0 = blockIdx.x * 16 * kQkFwdRows + hw;
  const __nv_bfloat16* src = qkv + static_cast<long long>(hh) * Dh + hl * 8;
  uint4 raw[kQkFwdRows];
#pragma unroll
  for (int i = 0; i < kQkFwdRows; ++i) {
    const int m = m0 + i * 16;
    raw[i] = m < M ? *reinterpret_cast<const uint4*>(src + m * rstride) : make_uint4(0, 0, 0, 0);
  }
  if (hh >= Hq + Hkv) {  // v head: copied through
    __nv_bfloat16* dst = v + static_cast<long long>(hh - Hq - Hkv) * Dh + hl * 8;
#pragma unroll
    for (int i = 0; i < kQkFwdRows; ++i) {
      const int m = m0 + i * 16;
      if (m < M) *reinterpret_cast<uint4*>(dst + static_cast<long long>(m) * Hkv * Dh) = raw[i];
    }
    return;
  }
  const bool is_q = hh < Hq;
  const int hsub = is_q ? hh : hh - Hq;
  const int nh = is_q ? Hq : Hkv;
  __nv_bfloat16* dst = (is_q ? q : k) + static_cast<long long>(hsub) * Dh + hl * 8;
  float* rdst = (is_q ? rq : rk) + hsub;
  float w[8];
  load_f32x8((is_q ? qs : ks) + hl * 8, w);
#pragma unroll
  for (int e = 0; e < 8; ++e) w[e] += 1.f;
#pragma unroll
  for (int i = 0; i < kQkFwdRows; ++i) {
    const int m = m0 + i * 16;
    float x[8];
    unpack_bf16x8(raw[i], x);
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += x[e] * x[e];
    const float r = rsqrtf(half_warp_sum(ss) / Dh + eps);
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] *= r * w[e];
    if (use_rope) {
      const int pos = start + ((m < M ? m : 0) % T);
      float c[8], sn[8];
      load_f32x8(cos_t + static_cast<long long>(pos) * 64 + (hl & 7) * 8, c);
      load_f32x8(sin_t + static_cast<long long>(pos) * 64 + (hl & 7) * 8, sn);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, x[e], 8);
        x[e] = hl < 8 ? x[e] * c[e] - partner * sn[e] : partner * sn[e] + x[e] * c[e];
      }
    }
    if (m < M) {
      *reinterpret_cast<uint4*>(dst + static_cast<long long>(m) * nh * Dh) = pack_bf16x8(x);
      if (hl == 0) rdst[static_cast<long long>(m) * nh] = r;
    }
  }
}

// Block (x, hh) handles head slot hh (a q, k or v head) of rows m = x*16*R + i*16 + hw, striding
// over m; every row is 256 contiguous bytes, so a fixed head per block costs no coalescing and
// gives each thread one kind of row: one set of scale weights and scale-gradient accumulators
// (its 8 columns), reduced once per block at the end.
template <int kQkBwdRows>
__global__ void __launch_bounds__(256, kQkBwdRows >= 4 ? 3 : 4) qk_norm_rope_bwd128_kernel(
    const __nv_bfloat16* __restrict__ dq, const __nv_bfloat16* __restrict__ dk, const __nv_bfloat16* __restrict__ dv,
    const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ rq, const float* __restrict__ rk,
    const float* __restrict__ qs, const float* __restrict__ ks, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, __nv_bfloat16* __restrict__ dqkv, float* __restrict__ dqs,
    float* __restrict__ dks, int M, int T, int Hq, int Hkv, int start, int use_rope) {
  constexpr int Dh = 128;
  __shared__ float s_acc[16][Dh];
  const int hw = threadIdx.x >> 4, hl = threadIdx.x & 15;
  const int hh = blockIdx.y;
  const int H = Hq + 2 * Hkv;
  const long long rstride = static_cast<long long>(H) * Dh;
  const int step = gridDim.x * 16 * kQkBwdRows;
  if (hh >= Hq + Hkv) {  // v head: the gradient passes through
    const __nv_bfloat16* src = dv + static_cast<long long>(hh - Hq - Hkv) * Dh + hl * 8;
    for (int m0 = blockIdx.x * 16 * kQkBwdRows; m0 < M; m0 += step) {
      uint4 g[kQkBwdRows];
#pragma unroll
      for (int i = 0; i < kQkBwdRows; ++i) {
        const int m = m0 + i * 16 + hw;
        g[i] = m < M ? *reinterpret_cast<const uint4*>(src + static_cast<long long>(m) * Hkv * Dh) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < kQkBwdRows; ++i) {
        const int m = m0 + i * 16 + hw;
        if (m < M) *reinterpret_cast<uint4*>(dqkv + m * rstride + static_cast<long long>(hh) * Dh + hl * 8) = g[i];
      }
    }
    return;
  }
  const bool is_q = hh < Hq;
  const int hsub = is_q ? hh : hh - Hq;
  const int nh = is_q ? Hq : Hkv;
  const __nv_bfloat16* gbase = (is_q ? dq : dk) + static_cast<long long>(hsub) * Dh + hl * 8;
  const float* rbase = (is_q ? rq : rk) + hsub;
  float w[8], acc[8];
  load_f32x8((is_q ? qs : ks) + hl * 8, w);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    w[e] += 1.f;
    acc[e] = 0.f;
  }
  for (int m0 = blockIdx.x * 16 * kQkBwdRows; m0 < M; m0 += step) {
    uint4 graw[kQkBwdRows], xraw[kQkBwdRows];
    float rr[kQkBwdRows];
#pragma unroll
    for (int i = 0; i < kQkBwdRows; ++i) {
      const int m = m0 + i * 16 + hw;
      const bool live = m < M;
      graw[i] = live ? *reinterpret_cast<const uint4*>(gbase + static_cast<long long>(m) * nh * Dh) : make_uint4(0, 0, 0, 0);
      xraw[i] = live ? *reinterpret_cast<const uint4*>(qkv + m * rstride + static_cast<long long>(hh) * Dh + hl * 8)
                     : make_uint4(0, 0, 0, 0);
      rr[i] = live ? rbase[static_cast<long long>(m) * nh] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < kQkBwdRows; ++i) {
      const int m = m0 + i * 16 + hw;
      float g[8], x[8];
      unpack_bf16x8(graw[i], g);
      unpack_bf16x8(xraw[i], x);
      if (use_rope) {
        const int pos = start + ((m < M ? m : 0) % T);
        float c[8], sn[8];
        load_f32x8(cos_t + static_cast<long long>(pos) * 64 + (hl & 7) * 8, c);
        load_f32x8(sin_t + static_cast<long long>(pos) * 64 + (hl & 7) * 8, sn);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float partner = __shfl_xor_sync(0xffffffffu, g[e], 8);
          g[e] = hl < 8 ? g[e] * c[e] + partner * sn[e] : -partner * sn[e] + g[e] * c[e];
        }
      }
      const float r = rr[i];
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) dot += g[e] * w[e] * x[e];
      dot = half_warp_sum(dot) / Dh;
      float d[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        d[e] = r * w[e] * g[e] - x[e] * r * r * r * dot;
        acc[e] += g[e] * x[e] * r;  // rows past M have g = 0
      }
      if (m < M) *reinterpret_cast<uint4*>(dqkv + m * rstride + static_cast<long long>(hh) * Dh + hl * 8) = pack_bf16x8(d);
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) s_acc[hw][hl * 8 + e] = acc[e];
  __syncthreads();
  if (threadIdx.x < Dh) {
    float t = 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) t += s_acc[r][threadIdx.x];
    atomicAdd((is_q ? dqs : dks) + threadIdx.x, t);
  }
}

__global__ void __launch_bounds__(256) qk_norm_rope_bwd_kernel(
    const __nv_bfloat16* __restrict__ dq, const __nv_bfloat16* __restrict__ dk, const __nv_bfloat16* __restrict__ dv,
    const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ rq, const float* __restrict__ rk,
    const float* __restrict__ qs, const float* __restrict__ ks, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, __nv_bfloat16* __restrict__ dqkv, float* __restrict__ dqs,
    float* __restrict__ dks, int M, int T, int Hq, int Hkv, int Dh, int start, int use_rope) {
  extern __shared__ float smem[];  // [8][Dh] grads + [8][2][Dh] per-warp scale accumulators
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* s_acc = smem + kRowsPerBlock * Dh;
  for (int j = threadIdx.x; j < kRowsPerBlock * 2 * Dh; j += blockDim.x) s_acc[j] = 0.f;
  __syncthreads();
  float* s_dq = s_acc + warp * 2 * Dh;
  float* s_dk = s_dq + Dh;
  const int H = Hq + 2 * Hkv;
  const long long total = static_cast<long long>(M) * H;
  const int half = Dh / 2;
  float* buf = smem + warp * Dh;
  for (long long item = static_cast<long long>(blockIdx.x) * kRowsPerBlock + warp; item < total;
       item += static_cast<long long>(gridDim.x) * kRowsPerBlock) {
    const int m = static_cast<int>(item / H);
    const int hh = static_cast<int>(item % H);
    __nv_bfloat16* out = dqkv + static_cast<long long>(m) * H * Dh + static_cast<long long>(hh) * Dh;
    if (hh >= Hq + Hkv) {
      const __nv_bfloat16* g = dv + (static_cast<long long>(m) * Hkv + (hh - Hq - Hkv)) * Dh;
      for (int j = lane; j < Dh; j += 32) out[j] = g[j];
      continue;
    }
    const bool is_q = hh < Hq;
    const __nv_bfloat16* g = is_q ? dq + (static_cast<long long>(m) * Hq + hh) * Dh
                                  : dk + (static_cast<long long>(m) * Hkv + (hh - Hq)) * Dh;
    const float* sc = is_q ? qs : ks;
    const float r = is_q ? rq[static_cast<long long>(m) * Hq + hh] : rk[static_cast<long long>(m) * Hkv + (hh - Hq)];
    const int pos = start + (m % T);
    // un-rotate the incoming gradient
    __syncwarp();
    for (int j = lane; j < Dh; j += 32) {
      float gn = __bfloat162float(g[j]);
      if (use_rope) {
        const int i = j < half ? j : j - half;
        const float c = cos_t[static_cast<long long>(pos) * half + i];
        const float s = sin_t[static_cast<long long>(pos) * half + i];
        gn = j < half ? __bfloat162float(g[j]) * c + __bfloat162float(g[j + half]) * s
                      : -__bfloat162float(g[j - half]) * s + __bfloat162float(g[j]) * c;
      }
      buf[j] = gn;
    }
    __syncwarp();
    const __nv_bfloat16* x = qkv + static_cast<long long>(m) * H * Dh + static_cast<long long>(hh) * Dh;
    float dot = 0.f;
    for (int j = lane; j < Dh; j += 32) dot += buf[j] * (1.f + sc[j]) * __bfloat162float(x[j]);
    dot = warp_sum(dot) / Dh;
    float* acc = is_q ? s_dq : s_dk;
    for (int j = lane; j < Dh; j += 32) {
      const float xv = __bfloat162float(x[j]);
      out[j] = __float2bfloat16_rn(r * (1.f + sc[j]) * buf[j] - xv * r * r * r * dot);
      acc[j] += buf[j] * xv * r;
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < Dh; j += blockDim.x) {
    float tq = 0.f, tk = 0.f;
    for (int w = 0; w < kRowsPerBlock; ++w) {
      tq += s_acc[w * 2 * Dh + j];
      tk += s_acc[w * 2 * Dh + Dh + j];
    }
    atomicAdd(&dqs[j], tq);
    atomicAdd(&dks[j], tk);
  }
}

int bwd_grid(int rows, int dev, int nwarps) {
  const int want = (rows + nwarps - 1) / nwarps;
  const int cap = num_sms(dev) * 4;
  return want < cap ? want : cap;
}

// warps per CTA such that nwarps * floats_per_warp fp32 accumulators fit in ~192 KB of shared memory
int bwd_warps(int floats_per_warp) {
  int w = 8;
  while (w > 1 && static_cast<long long>(w) * floats_per_warp * 4 > 192 * 1024) w >>= 1;
  return w;
}

}  // namespace

std::vector<at::Tensor> rmsnorm_fwd(const at::Tensor& x, const at::Tensor& scale, double eps, int64_t out_code) {
  check_contig(x, "x");
  check_contig(scale, "scale");
  MINT_CHECK(scale.scalar_type() == at::kFloat, "RMSNorm scale must be fp32");
  const int D = static_cast<int>(x.size(-1));
  const int rows = static_cast<int>(x.numel() / D);
  MINT_CHECK(scale.numel() == D, "scale size mismatch");
  const auto out_dt = out_code == 0 ? at::kFloat : (out_code == 1 ? at::kBFloat16 : at::kHalf);
  auto y = at::empty(x.sizes(), x.options().dtype(out_dt));
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  if (rows == 0) return {y, rstd};
  c10::cuda::CUDAGuard g(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
#define LAUNCH(TI, TO) \
  rmsnorm_fwd_kernel<TI, TO><<<grid, 256, 0, st>>>(reinterpret_cast<const TI*>(x.data_ptr()), scale.data_ptr<float>(), \
                                                  reinterpret_cast<TO*>(y.data_ptr()), rstd.data_ptr<float>(), rows, D, \
                                                  static_cast<float>(eps))
  if (x.scalar_type() == at::kFloat) {
    if (out_dt == at::kFloat) LAUNCH(float, float);
    else LAUNCH(float, __nv_bfloat16);
  } else {
    MINT_CHECK(x.scalar_type() == at::kBFloat16, "rmsnorm input must be fp32 or bf16");
    if (out_dt == at::kFloat) LAUNCH(__nv_bfloat16, float);
    else LAUNCH(__nv_bfloat16, __nv_bfloat16);
  }
#undef LAUNCH
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return {y, rstd};
}

std::vector<at::Tensor> rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& rstd,
                                    const at::Tensor& scale, int64_t dx_code) {
  check_contig(dy, "dy");
  check_contig(x, "x");
  const int D = static_cast<int>(x.size(-1));
  const int rows = static_cast<int>(x.numel() / D);
  MINT_CHECK(D <= kMaxD, "rmsnorm D too large");
  const auto dx_dt = dx_code == 0 ? at::kFloat : at::kBFloat16;
  auto dx = at::empty(x.sizes(), x.options().dtype(dx_dt));
  auto dscale = at::zeros({D}, x.options().dtype(at::kFloat));
  if (rows == 0) return {dx, dscale};
  c10::cuda::CUDAGuard g(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int nw = bwd_warps(D);
  const int grid = bwd_grid(rows, x.get_device(), nw);
  const size_t sm = static_cast<size_t>(nw) * D * sizeof(float);
  static bool attr_set = false;
  if (!attr_set) {
    MINT_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_bwd_kernel<float, float, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    MINT_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_bwd_kernel<float, __nv_bfloat16, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    MINT_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_bwd_kernel<__nv_bfloat16, __nv_bfloat16, __nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    MINT_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_bwd_kernel<__nv_bfloat16, float, __nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    MINT_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_bwd_kernel<float, __nv_bfloat16, __nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    MINT_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_bwd_kernel<__nv_bfloat16, __nv_bfloat16, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    MINT_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_bwd_kernel<float, float, __nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    MINT_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_bwd_kernel<__nv_bfloat16, float, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_set = true;
  }
#define LAUNCH(TI, TDY, TDX)                                                                                   \
  rmsnorm_bwd_kernel<TI, TDY, TDX><<<grid, nw * 32, sm, st>>>(                                                     \
      reinterpret_cast<const TDY*>(dy.data_ptr()), reinterpret_cast<const TI*>(x.data_ptr()), rstd.data_ptr<float>(), \
      scale.data_ptr<float>(), reinterpret_cast<TDX*>(dx.data_ptr()), dscale.data_ptr<float>(), rows, D)
  const bool xf = x.scalar_type() == at::kFloat, dyf = dy.scalar_type() == at::kFloat, dxf = dx_dt == at::kFloat;
  if (xf && !dyf && dxf && D % 256 == 0 && D <= 768) {
    const int grid_r = std::min<int>((rows + 7) / 8, num_sms(x.get_device()) * 2);
#define MINT_RMS_BWD_REG(VPT)                                                                                       \
  rmsnorm_bwd_reg_kernel<VPT><<<grid_r, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),        \
                                                      x.data_ptr<float>(), rstd.data_ptr<float>(), scale.data_ptr<float>(), \
                                                      dx.data_ptr<float>(), dscale.data_ptr<float>(), rows)
    switch (D / 32) {
      case 8: MINT_RMS_BWD_REG(8); break;
      case 16: MINT_RMS_BWD_REG(16); break;
      default: MINT_RMS_BWD_REG(24); break;
    }
#undef MINT_RMS_BWD_REG
    MINT_CUDA_CHECK(cudaGetLastError());
    count_launch();
    return {dx, dscale};
  }
  if (xf && dyf && dxf) LAUNCH(float, float, float);
  else if (xf && !dyf && dxf) LAUNCH(float, __nv_bfloat16, float);
  else if (!xf && !dyf && !dxf) LAUNCH(__nv_bfloat16, __nv_bfloat16, __nv_bfloat16);
  else if (!xf && dyf && !dxf) LAUNCH(__nv_bfloat16, float, __nv_bfloat16);
  else if (xf && !dyf && !dxf) LAUNCH(float, __nv_bfloat16, __nv_bfloat16);
  else if (!xf && !dyf && dxf) LAUNCH(__nv_bfloat16, __nv_bfloat16, float);
  else if (xf && dyf && !dxf) LAUNCH(float, float, __nv_bfloat16);
  else LAUNCH(__nv_bfloat16, float, float);
#undef LAUNCH
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return {dx, dscale};
}

std::vector<at::Tensor> add_rmsnorm_fwd(const at::Tensor& res, const at::Tensor& a, const at::Tensor& post,
                                        const c10::optional<at::Tensor>& pre, double eps, int64_t y_code) {
  check_contig(res, "res");
  check_contig(a, "a");
  MINT_CHECK(res.scalar_type() == at::kFloat && a.scalar_type() == at::kBFloat16, "add_rmsnorm: res fp32, a bf16");
  const int D = static_cast<int>(res.size(-1));
  const int rows = static_cast<int>(res.numel() / D);
  auto h = at::empty_like(res);
  const bool has_pre = pre.has_value() && pre->defined();
  const auto y_dt = y_code == 0 ? at::kFloat : at::kBFloat16;
  auto y = has_pre ? at::empty(res.sizes(), res.options().dtype(y_dt)) : at::empty({0}, res.options());
  auto ra = at::empty({rows}, res.options());
  auto rh = at::empty({has_pre ? rows : 0}, res.options());
  if (rows == 0) return {h, y, ra, rh};
  c10::cuda::CUDAGuard g(res.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  const float* pre_p = has_pre ? pre->data_ptr<float>() : nullptr;
  if (D % 256 == 0 && D <= 1024) {
    const __nv_bfloat16* ap = reinterpret_cast<const __nv_bfloat16*>(a.data_ptr());
#define MINT_ARN_FWD_REG(VPT)                                                                                    \
  if (y_dt == at::kFloat) {                                                                                      \
    add_rmsnorm_fwd_reg_kernel<VPT, float><<<grid, 256, 0, st>>>(                                               \
        res.data_ptr<float>(), ap, post.data_ptr<float>(), pre_p, h.data_ptr<float>(),                           \
        has_pre ? y.data_ptr<float>() : nullptr, ra.data_ptr<float>(), has_pre ? rh.data_ptr<float>() : nullptr, \
        rows, static_cast<float>(eps));                                                                          \
  } else {                                                                                                       \
    add_rmsnorm_fwd_reg_kernel<VPT, __nv_bfloat16><<<grid, 256, 0, st>>>(                                       \
        res.data_ptr<float>(), ap, post.data_ptr<float>(), pre_p, h.data_ptr<float>(),                           \
        has_pre ? reinterpret_cast<__nv_bfloat16*>(y.data_ptr()) : nullptr, ra.data_ptr<float>(),                \
        has_pre ? rh.data_ptr<float>() : nullptr, rows, static_cast<float>(eps));                                \
  }
    switch (D / 32) {
      case 8: MINT_ARN_FWD_REG(8); break;
      case 16: MINT_ARN_FWD_REG(16); break;
      case 24: MINT_ARN_FWD_REG(24); break;
      default: MINT_ARN_FWD_REG(32); break;
    }
#undef MINT_ARN_FWD_REG
  } else if (y_dt == at::kFloat) {
    add_rmsnorm_fwd_kernel<float><<<grid, 256, 0, st>>>(
        res.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(a.data_ptr()), post.data_ptr<float>(), pre_p,
        h.data_ptr<float>(), has_pre ? y.data_ptr<float>() : nullptr, ra.data_ptr<float>(),
        has_pre ? rh.data_ptr<float>() : nullptr, rows, D, static_cast<float>(eps));
  } else {
    add_rmsnorm_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        res.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(a.data_ptr()), post.data_ptr<float>(), pre_p,
        h.data_ptr<float>(), has_pre ? reinterpret_cast<__nv_bfloat16*>(y.data_ptr()) : nullptr, ra.data_ptr<float>(),
        has_pre ? rh.data_ptr<float>() : nullptr, rows, D, static_cast<float>(eps));
  }
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return {h, y, ra, rh};
}

std::vector<at::Tensor> add_rmsnorm_bwd(const c10::optional<at::Tensor>& dh, const c10::optional<at::Tensor>& dy,
                                        const at::Tensor& a, const at::Tensor& h, const at::Tensor& rstd_a,
                                        const at::Tensor& rstd_h, const at::Tensor& post,
                                        const c10::optional<at::Tensor>& pre) {
  check_contig(a, "a");
  check_contig(h, "h");
  const int D = static_cast<int>(h.size(-1));
  const int rows = static_cast<int>(h.numel() / D);
  MINT_CHECK(D <= kMaxD, "add_rmsnorm D too large");
  auto dres = at::empty_like(h);
  auto da = at::empty_like(a);
  auto dpost = at::zeros({D}, h.options());
  const bool has_pre = pre.has_value() && pre->defined();
  auto dpre = at::zeros({has_pre ? D : 0}, h.options());
  if (rows == 0) return {dres, da, dpost, dpre};
  c10::cuda::CUDAGuard g(h.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int nw = bwd_warps(2 * D);
  const int grid = bwd_grid(rows, h.get_device(), nw);
  const size_t sm = static_cast<size_t>(nw) * 2 * D * sizeof(float);
  static bool attr_set = false;
  if (!attr_set) {
    MINT_CUDA_CHECK(cudaFuncSetAttribute(add_rmsnorm_bwd_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    MINT_CUDA_CHECK(cudaFuncSetAttribute(add_rmsnorm_bwd_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_set = true;
  }
  const float* dh_p = (dh.has_value() && dh->defined()) ? dh->data_ptr<float>() : nullptr;
  const bool has_dy = dy.has_value() && dy->defined() && has_pre;
  if ((!has_dy || dy->scalar_type() == at::kBFloat16) && D % 256 == 0 && D <= 768) {
    // register-resident kernel: 4 warps per block, ~5 blocks per SM
    const int grid_r = std::min<int>((rows + kArnBwdWarps - 1) / kArnBwdWarps, num_sms(h.get_device()) * 5);
#define MINT_ARN_BWD_REG(VPT)                                                                                   \
  add_rmsnorm_bwd_reg_kernel<VPT><<<grid_r, kArnBwdWarps * 32, 0, st>>>(                                                     \
      dh_p, has_dy ? reinterpret_cast<const __nv_bfloat16*>(dy->data_ptr()) : nullptr,                          \
      reinterpret_cast<const __nv_bfloat16*>(a.data_ptr()), h.data_ptr<float>(), rstd_a.data_ptr<float>(),      \
      has_pre ? rstd_h.data_ptr<float>() : nullptr, post.data_ptr<float>(), has_pre ? pre->data_ptr<float>() : nullptr, \
      dres.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(da.data_ptr()), dpost.data_ptr<float>(),         \
      has_pre ? dpre.data_ptr<float>() : nullptr, rows)
    switch (D / 32) {
      case 8: MINT_ARN_BWD_REG(8); break;
      case 16: MINT_ARN_BWD_REG(16); break;
      default: MINT_ARN_BWD_REG(24); break;
    }
#undef MINT_ARN_BWD_REG
    MINT_CUDA_CHECK(cudaGetLastError());
    count_launch();
    return {dres, da, dpost, dpre};
  }
  if (!has_dy || dy->scalar_type() == at::kBFloat16) {
    add_rmsnorm_bwd_kernel<__nv_bfloat16><<<grid, nw * 32, sm, st>>>(
        dh_p, has_dy ? reinterpret_cast<const __nv_bfloat16*>(dy->data_ptr()) : nullptr,
        reinterpret_cast<const __nv_bfloat16*>(a.data_ptr()), h.data_ptr<float>(), rstd_a.data_ptr<float>(),
        has_pre ? rstd_h.data_ptr<float>() : nullptr, post.data_ptr<float>(), has_pre ? pre->data_ptr<float>() : nullptr,
        dres.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(da.data_ptr()), dpost.data_ptr<float>(),
        has_pre ? dpre.data_ptr<float>() : nullptr, rows, D);
  } else {
    add_rmsnorm_bwd_kernel<float><<<grid, nw * 32, sm, st>>>(
        dh_p, dy->data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(a.data_ptr()), h.data_ptr<float>(),
        rstd_a.data_ptr<float>(), rstd_h.data_ptr<float>(), post.data_ptr<float>(), pre->data_ptr<float>(),
        dres.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(da.data_ptr()), dpost.data_ptr<float>(),
        dpre.data_ptr<float>(), rows, D);
  }
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return {dres, da, dpost, dpre};
}

std::vector<at::Tensor> qk_norm_rope_fwd(const at::Tensor& qkv, int64_t n_q, int64_t n_kv, int64_t Dh,
                                         const at::Tensor& qs, const at::Tensor& ks, const at::Tensor& cos_t,
                                         const at::Tensor& sin_t, int64_t start, double eps, bool use_rope) {
  check_contig(qkv, "qkv");
  MINT_CHECK(qkv.dim() == 3 && qkv.scalar_type() == at::kBFloat16, "qkv must be [B, T, H*D] bf16");
  const int B = static_cast<int>(qkv.size(0)), T = static_cast<int>(qkv.size(1));
  MINT_CHECK(qkv.size(2) == (n_q + 2 * n_kv) * Dh, "qkv width mismatch");
  MINT_CHECK(Dh % 2 == 0 && Dh <= 1024, "head_dim must be even and <= 1024");
  if (use_rope) MINT_CHECK(cos_t.size(0) >= start + T && cos_t.size(1) == Dh / 2, "rope table too small");
  const int M = B * T;
  auto opts = qkv.options();
  auto q = at::empty({B, T, n_q, Dh}, opts);
  auto k = at::empty({B, T, n_kv, Dh}, opts);
  auto v = at::empty({B, T, n_kv, Dh}, opts);
  auto rq = at::empty({M, n_q}, opts.dtype(at::kFloat));
  auto rk = at::empty({M, n_kv}, opts.dtype(at::kFloat));
  const long long items = static_cast<long long>(M) * (n_q + 2 * n_kv);
  if (items == 0) return {q, k, v, rq, rk};
  c10::cuda::CUDAGuard g(qkv.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = static_cast<int>((items + kRowsPerBlock - 1) / kRowsPerBlock);
  if (Dh == 128) {
    const dim3 grid128(static_cast<unsigned>((M + 16 * kQkFwdRows - 1) / (16 * kQkFwdRows)),
                       static_cast<unsigned>(n_q + 2 * n_kv));
    qk_norm_rope_fwd128_kernel<<<grid128, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qs.data_ptr<float>(), ks.data_ptr<float>(),
        cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(q.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(k.data_ptr()), reinterpret_cast<__nv_bfloat16*>(v.data_ptr()),
        rq.data_ptr<float>(), rk.data_ptr<float>(), M, T, static_cast<int>(n_q), static_cast<int>(n_kv),
        static_cast<int>(start), use_rope ? 1 : 0, static_cast<float>(eps));
    MINT_CUDA_CHECK(cudaGetLastError());
    count_launch();
    return {q, k, v, rq, rk};
  }
  qk_norm_rope_fwd_kernel<<<grid, 256, kRowsPerBlock * Dh * sizeof(float), st>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qs.data_ptr<float>(), ks.data_ptr<float>(),
      cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(q.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(k.data_ptr()), reinterpret_cast<__nv_bfloat16*>(v.data_ptr()),
      rq.data_ptr<float>(), rk.data_ptr<float>(), M, T, static_cast<int>(n_q), static_cast<int>(n_kv),
      static_cast<int>(Dh), static_cast<int>(start), use_rope ? 1 : 0, static_cast<float>(eps));
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return {q, k, v, rq, rk};
}

std::vector<at::Tensor> qk_norm_rope_bwd(const at::Tensor& dq, const at::Tensor& dk, const at::Tensor& dv,
                                         const at::Tensor& qkv, const at::Tensor& rq, const at::Tensor& rk,
                                         const at::Tensor& qs, const at::Tensor& ks, const at::Tensor& cos_t,
                                         const at::Tensor& sin_t, int64_t n_q, int64_t n_kv, int64_t Dh,
                                         int64_t start, bool use_rope) {
  check_contig(dq, "dq");
  check_contig(dk, "dk");
  check_contig(dv, "dv");
  MINT_CHECK(dq.scalar_type() == at::kBFloat16 && dk.scalar_type() == at::kBFloat16 &&
                 dv.scalar_type() == at::kBFloat16, "qk_norm_rope_bwd expects bf16 grads");
  const int B = static_cast<int>(qkv.size(0)), T = static_cast<int>(qkv.size(1));
  const int M = B * T;
  auto dqkv = at::empty_like(qkv);
  auto dqs = at::zeros({Dh}, qkv.options().dtype(at::kFloat));
  auto dks = at::zeros({Dh}, qkv.options().dtype(at::kFloat));
  const long long items = static_cast<long long>(M) * (n_q + 2 * n_kv);
  if (items == 0) return {dqkv, dqs, dks};
  c10::cuda::CUDAGuard g(qkv.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const long long want = (items + kRowsPerBlock - 1) / kRowsPerBlock;
  const long long cap = static_cast<long long>(num_sms(qkv.get_device())) * 8;
  const int grid = static_cast<int>(want < cap ? want : cap);
  if (Dh == 128) {
    const int H = static_cast<int>(n_q + 2 * n_kv);
    static const int rows_env = [] {
      const char* e = std::getenv("MINT_QK_BWD_ROWS");
      return e != nullptr && std::atoi(e) == 2 ? 2 : 4;
    }();
    const long long gx_want = (M + 16 * rows_env - 1) / (16 * rows_env);
    const long long gx_cap = std::max<long long>(1, (static_cast<long long>(num_sms(qkv.get_device())) * 8 + H - 1) / H);
    const dim3 grid128(static_cast<unsigned>(std::min(gx_want, gx_cap)), static_cast<unsigned>(H));
    auto kern = rows_env == 2 ? qk_norm_rope_bwd128_kernel<2> : qk_norm_rope_bwd128_kernel<4>;
    kern<<<grid128, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(dq.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dk.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(dv.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
        rq.data_ptr<float>(), rk.data_ptr<float>(), qs.data_ptr<float>(), ks.data_ptr<float>(),
        cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()),
        dqs.data_ptr<float>(), dks.data_ptr<float>(), M, T, static_cast<int>(n_q), static_cast<int>(n_kv),
        static_cast<int>(start), use_rope ? 1 : 0);
    MINT_CUDA_CHECK(cudaGetLastError());
    count_launch();
    return {dqkv, dqs, dks};
  }
  qk_norm_rope_bwd_kernel<<<grid, 256, 3 * kRowsPerBlock * Dh * sizeof(float), st>>>(
      reinterpret_cast<const __nv_bfloat16*>(dq.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dk.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(dv.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
      rq.data_ptr<float>(), rk.data_ptr<float>(), qs.data_ptr<float>(), ks.data_ptr<float>(),
      cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()),
      dqs.data_ptr<float>(), dks.data_ptr<float>(), M, T, static_cast<int>(n_q), static_cast<int>(n_kv),
      static_cast<int>(Dh), static_cast<int>(start), use_rope ? 1 : 0);
  MINT_CUDA_CHECK(cudaGetLastError());
  count_launch();
  return {dqkv, dqs, dks};
}

}  // namespace mint
